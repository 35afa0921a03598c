"""Generate the golden vectors under tests/golden/ from the reference itself.

Run in a container where the reference sources are mounted, with
KINETIC_REFERENCE naming the reference's root directory:

    KINETIC_REFERENCE=<reference root> python tests/golden/make_golden.py

It imports the reference's own PyTorch parity functions
(tests/test_fusion.py:11-51) and its Triton kernel
(python/kinetic_rt/fusion_forge.py:21-162, run under TRITON_INTERPRET=1),
evaluates them on seeded inputs and writes .npz fixtures.  The fixtures are
what the oracle and the CUDA path are checked against; nothing at test time
reads the reference tree.

Inputs other than the known-answer case are drawn from numpy's PCG64 by
tests/golden/inputs.py, so tests can regenerate them; each fixture stores a
sha256 of its inputs to pin that generator.
"""
import hashlib
import importlib.util
import os
import sys
import types

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from tests.golden import inputs as golden_inputs  # noqa: E402
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits  # noqa: E402

REF = os.environ.get("KINETIC_REFERENCE", "")


def _load_reference():
    """Import fusion_forge and test_fusion from the reference tree without
    executing the package __init__ (which needs the compiled _core)."""
    pkg = types.ModuleType("python")
    pkg.__path__ = [os.path.join(REF, "python")]
    sub = types.ModuleType("python.kinetic_rt")
    sub.__path__ = [os.path.join(REF, "python", "kinetic_rt")]
    sys.modules["python"] = pkg
    sys.modules["python.kinetic_rt"] = sub
    import python.kinetic_rt.fusion_forge as ff  # noqa: E402
    spec = importlib.util.spec_from_file_location("ref_test_fusion", os.path.join(REF, "tests", "test_fusion.py"))
    tf = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tf)
    return ff, tf


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def known_answer(ff, tf):
    """tests/test_fusion.py:65-121 verbatim inputs (seed 42, B=S=1, d=128)."""
    torch.manual_seed(42)
    d = 128
    x = torch.randn(1, 1, d, dtype=torch.float32)
    rms_w = torch.ones(d, dtype=torch.float32)
    w = torch.randn(3 * d, d, dtype=torch.float32)
    cos = torch.randn(1, 1, d, dtype=torch.float32)
    sin = torch.randn(1, 1, d, dtype=torch.float32)
    rq, rk, rv = tf.run_pytorch_reference(x, w, rms_w, cos, sin, d)
    tq, tk, tv = torch.empty_like(rq), torch.empty_like(rk), torch.empty_like(rv)
    ff.fused_rmsnorm_qkv_rope[(1,)](
        x, w, None, rms_w, cos, sin, tq, tk, tv, 1, d, 1, d, 1e-5,
        x.stride(1), x.stride(2), w.stride(0), w.stride(1),
        tq.stride(1), tq.stride(2), tk.stride(1), tk.stride(2), tv.stride(1), tv.stride(2),
        BLOCK_DIM=128)
    np.savez_compressed(
        os.path.join(HERE, "known_answer_d128.npz"),
        x=x.numpy(), rms_w=rms_w.numpy(), w=w.numpy(), cos=cos.numpy(), sin=sin.numpy(),
        ref_q=rq.numpy(), ref_k=rk.numpy(), ref_v=rv.numpy(),
        triton_q=tq.numpy(), triton_k=tk.numpy(), triton_v=tv.numpy())
    print("known_answer_d128: triton vs torch max-abs",
          float((tq - rq).abs().max()), float((tk - rk).abs().max()), float((tv - rv).abs().max()))


def per_head_reference(tf, x, w, g, cos, sin, nh, nkv, hd, bias=None):
    """run_pytorch_reference's pieces composed per head (rope_ref on
    [..., H, hd] views), GQA split [Q | K | V]."""
    xn = tf.rms_norm_ref(x, g)
    qkv = tf.qkv_linear_ref(xn, w, bias)
    nq, nk = nh * hd, nkv * hd
    lead = qkv.shape[:-1]
    q = qkv[..., :nq].reshape(*lead, nh, hd)
    k = qkv[..., nq:nq + nk].reshape(*lead, nkv, hd)
    v = qkv[..., nq + nk:].reshape(*lead, nkv, hd)
    q, k = tf.rope_ref(q, k, cos.unsqueeze(-2), sin.unsqueeze(-2))
    return q, k, v


def config1(tf):
    """Batch 2, seq 32, hidden 512, 8 Q / 8 KV heads x 64, fp32, theta 1e4."""
    c = golden_inputs.config1_inputs()
    x, w, g, cos, sin = (torch.from_numpy(c[n]) for n in ("x", "w", "gamma", "cos", "sin"))
    q, k, v = per_head_reference(tf, x, w, g, cos, sin, 8, 8, 64)
    # The literal whole-row call of tests/test_fusion.py:48, for the record.
    lq, lk, lv = tf.run_pytorch_reference(x, w, g, cos.repeat(1, 1, 8)[..., :512], sin.repeat(1, 1, 8)[..., :512], 512)
    np.savez_compressed(
        os.path.join(HERE, "config1_fp32.npz"),
        inputs_sha256=np.array(sha(*(c[n] for n in sorted(c)))),
        q=q.numpy(), k=k.numpy(), v=v.numpy(),
        literal_q_maxdiff=np.array(float((lq.reshape(q.shape) - q).abs().max())))
    print("config1_fp32: per-head vs literal whole-row RoPE max-abs", float((lq.reshape(q.shape) - q).abs().max()))


def gqa_bf16(tf):
    """Small Llama-shaped bf16 case with GQA, ragged positions and bias."""
    c = golden_inputs.gqa_bf16_inputs()
    f = {n: torch.from_numpy(bf16_bits_to_f32(c[n])) for n in ("x", "w", "gamma", "bias")}
    cos, sin = torch.from_numpy(c["cos"]), torch.from_numpy(c["sin"])
    nh, nkv, hd = c["dims"].tolist()
    # fp32 evaluation on the bf16 input values, with the normalised activation
    # rounded to bf16 as the fused kernel does (fusion_forge.py:47).
    xn = tf.rms_norm_ref(f["x"], f["gamma"]).to(torch.bfloat16).float()
    qkv = tf.qkv_linear_ref(xn, f["w"], f["bias"])
    nq, nk = nh * hd, nkv * hd
    q = qkv[..., :nq].reshape(-1, nh, hd)
    k = qkv[..., nq:nq + nk].reshape(-1, nkv, hd)
    v = qkv[..., nq + nk:].reshape(-1, nkv, hd)
    q, k = tf.rope_ref(q, k, cos.unsqueeze(-2), sin.unsqueeze(-2))
    # The same reference functions run literally in bf16 arithmetic.
    xb = {n: t.to(torch.bfloat16) for n, t in f.items()}
    bq, bk, bv = per_head_reference(tf, xb["x"], xb["w"], xb["gamma"], cos.to(torch.bfloat16),
                                    sin.to(torch.bfloat16), nh, nkv, hd, bias=xb["bias"])
    np.savez_compressed(
        os.path.join(HERE, "gqa_bf16.npz"),
        inputs_sha256=np.array(sha(*(c[n] for n in sorted(c)))),
        q=q.numpy(), k=k.numpy(), v=v.numpy(),
        bf16_q=f32_to_bf16_bits(bq.float().numpy()), bf16_k=f32_to_bf16_bits(bk.float().numpy()),
        bf16_v=f32_to_bf16_bits(bv.float().numpy()))
    print("gqa_bf16: literal-bf16 reference vs fp32 evaluation max-abs",
          float((bq.float() - q).abs().max()), float((bk.float() - k).abs().max()))


if __name__ == "__main__":
    if not REF or not os.path.isdir(os.path.join(REF, "python", "kinetic_rt")):
        sys.exit("set KINETIC_REFERENCE to the reference's root directory")
    ff, tf = _load_reference()
    known_answer(ff, tf)
    config1(tf)
    gqa_bf16(tf)
