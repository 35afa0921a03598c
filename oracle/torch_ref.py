"""The reference's CPU path for the decoder hot path, in torch (test and
baseline infrastructure only: bench.py times it as the CPU baseline).

Restates tests/test_fusion.py:11-51 (rms_norm_ref, qkv_linear_ref, rope_ref,
run_pytorch_reference) with RoPE applied per head and a GQA split, plus the
fp32 row-parallel products of o_proj and down_proj (scripts/export_hf.py:
62-65 shards, summed as the allreduce would).  Runs in fp32 on the host's
cores, as the reference does.
"""
import torch
import torch.nn.functional as F


def rms_norm_ref(x, weight, eps=1e-5):
    variance = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(variance + eps) * weight


def rotate_half(x):
    x1, x2 = x[..., :x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def qkv_rope_ref(x, w_qkv, gamma, cos, sin, n_heads, n_kv_heads, head_dim, eps=1e-5):
    """x [T, D]; cos/sin [T, hd] (rows at each token's position)."""
    qkv = F.linear(rms_norm_ref(x, gamma, eps), w_qkv)
    nq, nk = n_heads * head_dim, n_kv_heads * head_dim
    q = qkv[:, :nq].view(-1, n_heads, head_dim)
    k = qkv[:, nq:nq + nk].view(-1, n_kv_heads, head_dim)
    v = qkv[:, nq + nk:]
    c, s = cos[:, None, :], sin[:, None, :]
    return q * c + rotate_half(q) * s, k * c + rotate_half(k) * s, v


def layer_hot_path_ref(x, w_qkv, gamma, cos, sin, attn_out, w_o, mlp_act, w_down, n_heads, n_kv_heads, head_dim):
    """One decoder layer's hot path on the CPU: fused QKV + RoPE, o_proj and
    down_proj (the unsharded products equal the allreduced shards)."""
    q, k, v = qkv_rope_ref(x, w_qkv, gamma, cos, sin, n_heads, n_kv_heads, head_dim)
    y_o = F.linear(attn_out, w_o)
    y_d = F.linear(mlp_act, w_down)
    return q, k, v, y_o, y_d
