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


def decode_layer_ref(h, w_qkv, g_attn, cos, sin, k_cache, v_cache, w_o, g_mlp, w_gate, w_up, w_down,
                     n_heads, n_kv_heads, head_dim, eps=1e-5):
    """One Llama decoder layer for one new token per sequence, on the CPU in
    fp32: RMSNorm + QKV + RoPE (tests/test_fusion.py:11-51 per head), attention
    over the cached K/V plus the new token's, o_proj + residual, RMSNorm,
    SwiGLU MLP + residual.  h [B, D]; k_cache / v_cache [B, ctx, Hkv, hd]."""
    q, k, v = qkv_rope_ref(h, w_qkv, g_attn, cos, sin, n_heads, n_kv_heads, head_dim, eps)
    B = h.shape[0]
    kk = torch.cat([k_cache, k[:, None]], 1)  # [B, ctx + 1, Hkv, hd]
    vv = torch.cat([v_cache, v.view(B, 1, n_kv_heads, head_dim)], 1)
    rep = n_heads // n_kv_heads
    kk = kk.permute(0, 2, 1, 3).repeat_interleave(rep, 1)  # [B, H, ctx + 1, hd]
    vv = vv.permute(0, 2, 1, 3).repeat_interleave(rep, 1)
    a = F.scaled_dot_product_attention(q[:, :, None, :], kk, vv)[:, :, 0, :].reshape(B, -1)
    h = h + F.linear(a, w_o)
    x = rms_norm_ref(h, g_mlp, eps)
    return h + F.linear(F.silu(F.linear(x, w_gate)) * F.linear(x, w_up), w_down)


def lm_head_greedy_ref(h, g_final, w_lm, eps=1e-5):
    """Final RMSNorm, lm_head and the greedy choice (python/kinetic_rt/
    orchestrator.py:442-444: argmax of the last token's logits)."""
    return torch.argmax(F.linear(rms_norm_ref(h, g_final, eps), w_lm), dim=-1)
