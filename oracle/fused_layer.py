"""Oracle for the fused RMSNorm + QKV projection + RoPE layer (test infrastructure).

Restates, in numpy, the reference's parity definition:

  rms_norm_ref          tests/test_fusion.py:11-14
      x * rsqrt(mean(x^2, -1) + eps) * weight
  qkv_linear_ref        tests/test_fusion.py:16-19
      F.linear(x, W, b)  with W in (out_features, in_features) layout
  rope_ref              tests/test_fusion.py:21-32
      u * cos + rotate_half(u) * sin,  rotate_half(u) = cat(-u2, u1)
  run_pytorch_reference tests/test_fusion.py:34-51
      q, k, v = qkv[..., :d], qkv[..., d:2d], qkv[..., 2d:]; v is not rotated

and the fused Triton kernel's order of operations
(python/kinetic_rt/fusion_forge.py:21-162): the normalised activation is
cast back to the input dtype before the projection (line 47), the
projection and RoPE run in fp32 (lines 57-139), and the stores cast to the
output dtype (lines 155-162).

RoPE is applied per head: ``rope_ref`` is evaluated on ``[..., H, head_dim]``
views with cos/sin broadcast over heads.  With one head of width d_model this
is exactly the literal reference call of tests/test_fusion.py:48 (and the
Triton kernel's whole-row rotation, fusion_forge.py:101-139).  Grouped-query
attention splits the projection rows as [Q heads | K heads | V heads].
"""
import numpy as np

from .bf16 import round_bf16


def rms_norm(x, weight, eps=1e-5):
    """tests/test_fusion.py:11-14, evaluated in fp32."""
    x = np.asarray(x, dtype=np.float32)
    var = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    r = (1.0 / np.sqrt(var + eps)).astype(np.float32)
    return (x * r * np.asarray(weight, dtype=np.float32)).astype(np.float32)


def qkv_linear(xn, w, b=None):
    """tests/test_fusion.py:16-19: F.linear(x, W, b), accumulated in fp64."""
    out = np.asarray(xn, np.float64) @ np.asarray(w, np.float64).T
    if b is not None:
        out = out + np.asarray(b, np.float64)
    return out.astype(np.float32)


def rotate_half(u):
    """tests/test_fusion.py:25-27."""
    h = u.shape[-1] // 2
    return np.concatenate((-u[..., h:], u[..., :h]), axis=-1)


def rope(u, cos, sin):
    """tests/test_fusion.py:29-30 for one tensor."""
    return (u * cos + rotate_half(u) * sin).astype(np.float32)


def fused_layer(x, w, gamma, cos, sin, n_heads, n_kv_heads, head_dim,
                bias=None, eps=1e-5, act_dtype="f32"):
    """RMSNorm -> QKV projection -> per-head RoPE on Q and K.

    x      [..., D] activations (float32 values; bf16 inputs already expanded)
    w      [(Hq + 2*Hkv) * hd, D] fused projection weight, Linear layout
    gamma  [D] RMSNorm weight
    cos, sin  broadcastable to [..., hd] (one table row per token, shared by
           all heads) or to [..., H, hd] (one row per token and head)
    act_dtype "f32" or "bf16": the dtype the normalised activation is cast
           to before the projection (fusion_forge.py:47).

    Returns fp32 (q [..., Hq, hd], k [..., Hkv, hd], v [..., Hkv, hd]).
    """
    xn = rms_norm(x, gamma, eps)
    if act_dtype == "bf16":
        xn = round_bf16(xn)
    qkv = qkv_linear(xn, w, bias)
    lead = qkv.shape[:-1]
    nq, nk = n_heads * head_dim, n_kv_heads * head_dim
    q = qkv[..., :nq].reshape(*lead, n_heads, head_dim)
    k = qkv[..., nq:nq + nk].reshape(*lead, n_kv_heads, head_dim)
    v = qkv[..., nq + nk:nq + 2 * nk].reshape(*lead, n_kv_heads, head_dim)
    c = np.asarray(cos, np.float32)
    s = np.asarray(sin, np.float32)
    if c.ndim == len(lead) + 1:           # one row per token -> broadcast over heads
        c = c[..., None, :]
        s = s[..., None, :]
    q = rope(q, c, s)
    k = rope(k, c[..., :1, :] if c.shape[-2] == 1 else c[..., :n_kv_heads, :],
             s[..., :1, :] if s.shape[-2] == 1 else s[..., :n_kv_heads, :])
    return q, k, v


def literal_reference(x, w, gamma, cos, sin, d_model, bias=None, eps=1e-5):
    """run_pytorch_reference (tests/test_fusion.py:34-51) taken literally:
    MHA split at d_model and RoPE over the whole last dimension."""
    xn = rms_norm(x, gamma, eps)
    qkv = qkv_linear(xn, w, bias)
    q, k, v = qkv[..., :d_model], qkv[..., d_model:2 * d_model], qkv[..., 2 * d_model:]
    return rope(q, cos, sin), rope(k, cos, sin), v


def rope_tables(positions, head_dim, theta):
    """Llama rotary tables: emb = cat(pos * inv_freq, pos * inv_freq),
    inv_freq = theta ** (-2i / head_dim).  Returns fp32 (cos, sin) of shape
    [len(positions), head_dim], computed in fp64 then rounded."""
    i = np.arange(0, head_dim, 2, dtype=np.float64)
    inv_freq = 1.0 / (theta ** (i / head_dim))
    f = np.outer(np.asarray(positions, np.float64), inv_freq)
    emb = np.concatenate([f, f], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
