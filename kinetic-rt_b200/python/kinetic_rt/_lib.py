"""ctypes binding of libkrt.so, the C ABI declared in include/krt.h.

This is the thinnest possible layer: struct mirrors, argument marshalling
from torch tensors (data_ptr / strides / current stream) and error
translation.  Every argument struct built here keeps references to the
tensors whose raw pointers it holds (`_refs`), so a struct kept for later
launches (or captured into a CUDA graph) cannot outlive its tensors.  Loading fails loudly when the library is missing; there is no
fallback implementation.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkrt.so")

KRT_OK = 0
KRT_ERR_INVALID = 1
KRT_ERR_CUDA = 2
KRT_ERR_UNSUPPORTED = 3
KRT_ERR_WORKSPACE = 4
KRT_ERR_DEVICE = 5
KRT_DTYPE_FLOAT32 = 1
KRT_DTYPE_BFLOAT16 = 3

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class QkvRopeArgs(ctypes.Structure):
    """krt_qkv_rope_args"""
    _fields_ = [
        ("x", _vp), ("qkv_weight", _vp), ("qkv_bias", _vp), ("rms_weight", _vp),
        ("freqs_cos", _vp), ("freqs_sin", _vp), ("q_out", _vp), ("k_out", _vp), ("v_out", _vp),
        ("seq_len", _i32), ("d_model", _i32), ("n_heads", _i32), ("head_dim", _i32),
        ("eps", ctypes.c_float),
        ("stride_x_seq", _i64), ("stride_x_dim", _i64), ("stride_w_out", _i64), ("stride_w_in", _i64),
        ("stride_q_seq", _i64), ("stride_q_dim", _i64), ("stride_k_seq", _i64), ("stride_k_dim", _i64),
        ("stride_v_seq", _i64), ("stride_v_dim", _i64),
        ("dtype", _i32), ("n_kv_heads", _i32), ("freqs_dtype", _i32), ("freqs_head_stride", _i32),
        ("stride_f_seq", _i64), ("stride_f_dim", _i64), ("positions", _vp),
    ]


class QkvPagedArgs(ctypes.Structure):
    """krt_qkv_paged_args"""
    _fields_ = [
        ("x", _vp), ("qkv_weight", _vp), ("qkv_bias", _vp), ("rms_weight", _vp),
        ("rope_cos", _vp), ("rope_sin", _vp), ("positions", _vp), ("token_seq", _vp),
        ("block_table", _vp), ("kv_pool", _vp), ("q_out", _vp), ("k_out", _vp), ("v_out", _vp),
        ("num_tokens", _i32), ("d_model", _i32), ("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32),
        ("x_stride", _i32), ("q_stride", _i32), ("max_position", _i32),
        ("num_seqs", _i32), ("block_table_stride", _i32), ("num_blocks", _i32), ("tokens_per_block", _i32),
        ("eps", ctypes.c_float), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class GemmArArgs(ctypes.Structure):
    """krt_gemm_ar_args"""
    _fields_ = [
        ("x", _vp), ("weight", _vp), ("y", _vp),
        ("num_tokens", _i32), ("k_local", _i32), ("n_out", _i32), ("x_stride", _i32), ("y_stride", _i32),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t), ("residual", _vp),
    ]


class PagedAttentionArgs(ctypes.Structure):
    """krt_paged_attention_args"""
    _fields_ = [
        ("q", _vp), ("kv_pool", _vp), ("block_table", _vp), ("seq_lens", _vp), ("out", _vp),
        ("num_seqs", _i32), ("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32),
        ("q_stride", _i32), ("out_stride", _i32),
        ("block_table_stride", _i32), ("num_blocks", _i32), ("tokens_per_block", _i32),
        ("max_seq_len", _i32), ("scale", ctypes.c_float),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class PagedPrefillAttentionArgs(ctypes.Structure):
    """krt_paged_prefill_attention_args"""
    _fields_ = [
        ("q", _vp), ("out", _vp), ("kv_pool", _vp), ("block_table", _vp), ("q_start", _vp), ("q_pos0", _vp),
        ("num_seqs", _i32), ("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32),
        ("q_stride", _i32), ("out_stride", _i32),
        ("block_table_stride", _i32), ("num_blocks", _i32), ("tokens_per_block", _i32),
        ("max_q_len", _i32), ("scale", ctypes.c_float),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class GateUpArgs(ctypes.Structure):
    """krt_gate_up_args"""
    _fields_ = [
        ("x", _vp), ("rms_weight", _vp), ("gate_up_weight", _vp), ("act", _vp),
        ("num_tokens", _i32), ("d_model", _i32), ("inter_local", _i32), ("x_stride", _i32), ("act_stride", _i32),
        ("eps", ctypes.c_float), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class LmHeadArgs(ctypes.Structure):
    """krt_lm_head_args"""
    _fields_ = [
        ("x", _vp), ("rms_weight", _vp), ("weight", _vp), ("argmax_keys", _vp),
        ("num_tokens", _i32), ("d_model", _i32), ("vocab_local", _i32), ("vocab_offset", _i32), ("x_stride", _i32),
        ("eps", ctypes.c_float), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class GreedyStepArgs(ctypes.Structure):
    """krt_greedy_step_args"""
    _fields_ = [
        ("argmax_keys", _vp), ("tokens", _vp), ("embedding", _vp), ("hidden", _vp),
        ("positions", _vp), ("seq_lens", _vp),
        ("num_seqs", _i32), ("d_model", _i32), ("hidden_stride", _i32), ("vocab", _i32),
        ("status", _vp), ("next_input", _vp),
    ]


# Every symbol include/krt.h declares, with (restype, argtypes).
SIGNATURES = {
    "krt_last_error": (ctypes.c_char_p, []),
    "krt_version": (ctypes.c_char_p, []),
    "krt_fused_rmsnorm_qkv_rope": (ctypes.c_int, [ctypes.POINTER(QkvRopeArgs), _vp]),
    "krt_qkv_rope_decode_workspace_size": (ctypes.c_size_t, [_i32, _i32, _i32, _i32, _i32]),
    "krt_qkv_rope_decode": (ctypes.c_int, [ctypes.POINTER(QkvPagedArgs), _vp]),
    "krt_qkv_rope_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(QkvPagedArgs), _vp]),
    "krt_qkv_rope_decode_noalloc_status": (ctypes.c_int, [_vp, ctypes.POINTER(_i32)]),
    "krt_qkv_rope_prefill_workspace_size": (ctypes.c_size_t, [_i32, _i32, _i32, _i32, _i32]),
    "krt_qkv_rope_prefill": (ctypes.c_int, [ctypes.POINTER(QkvPagedArgs), _vp]),
    "krt_read_status": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(_i32)]),
    "krt_comm_create": (ctypes.c_int, [_i32, _i32, _i32, ctypes.POINTER(_vp)]),
    "krt_comm_handle_size": (ctypes.c_size_t, []),
    "krt_comm_ipc_handle": (ctypes.c_int, [_vp, _vp]),
    "krt_comm_open_peers": (ctypes.c_int, [_vp, _vp]),
    "krt_comm_destroy": (ctypes.c_int, [_vp]),
    "krt_comm_reset": (ctypes.c_int, [_vp, _vp]),
    "krt_nccl_id_size": (ctypes.c_size_t, []),
    "krt_nccl_unique_id": (ctypes.c_int, [_vp]),
    "krt_comm_attach_nccl": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t]),
    "krt_allreduce": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_size_t, _i32, _vp, _vp]),
    "krt_rowparallel_gemm_ar_workspace_size": (ctypes.c_size_t, []),
    "krt_rowparallel_gemm_ar": (ctypes.c_int, [_vp, ctypes.POINTER(GemmArArgs), _vp]),
    "krt_paged_attention_workspace_size": (ctypes.c_size_t, [_i32, _i32, _i32, _i32]),
    "krt_paged_attention_decode": (ctypes.c_int, [ctypes.POINTER(PagedAttentionArgs), _vp]),
    "krt_paged_attention_prefill_workspace_size": (ctypes.c_size_t, []),
    "krt_paged_attention_prefill": (ctypes.c_int, [ctypes.POINTER(PagedPrefillAttentionArgs), _vp]),
    "krt_projection_workspace_size": (ctypes.c_size_t, [_i32, _i32]),
    "krt_gate_up_swiglu": (ctypes.c_int, [ctypes.POINTER(GateUpArgs), _vp]),
    "krt_lm_head_argmax": (ctypes.c_int, [ctypes.POINTER(LmHeadArgs), _vp]),
    "krt_greedy_step": (ctypes.c_int, [_vp, ctypes.POINTER(GreedyStepArgs), _vp]),
}

_lib = None


def lib():
    """Load libkrt.so once.  Raises ImportError when it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libkrt.so not found at {LIB_PATH}; run kinetic-rt_b200/build.py")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


class KrtError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def check(rc):
    if rc != KRT_OK:
        msg = lib().krt_last_error().decode()
        if rc in (KRT_ERR_INVALID, KRT_ERR_UNSUPPORTED, KRT_ERR_WORKSPACE):
            err = ValueError(msg)
            err.code = rc
            raise err
        raise KrtError(rc, msg)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is not None:
        return ctypes.c_void_p(int(stream))
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dtype_code(t):
    import torch
    if t.dtype == torch.float32:
        return KRT_DTYPE_FLOAT32
    if t.dtype == torch.bfloat16:
        return KRT_DTYPE_BFLOAT16
    raise ValueError(f"unsupported dtype {t.dtype}; float32 and bfloat16 are supported")


def fused_rmsnorm_qkv_rope(x, qkv_weight, qkv_bias, rms_weight, freqs_cos, freqs_sin, q_out, k_out, v_out,
                           seq_len, d_model, n_heads, head_dim, eps, strides, n_kv_heads=0,
                           freqs_strides=None, freqs_head_stride=-1, positions=None, stream=None):
    """Generic CUDA-core path (krt_fused_rmsnorm_qkv_rope) on device tensors.
    `strides` = the reference's ten strides in argument order
    (fusion_forge.py:26-30)."""
    a = QkvRopeArgs()
    a.x, a.qkv_weight, a.qkv_bias, a.rms_weight = _ptr(x), _ptr(qkv_weight), _ptr(qkv_bias), _ptr(rms_weight)
    a.freqs_cos, a.freqs_sin = _ptr(freqs_cos), _ptr(freqs_sin)
    a.q_out, a.k_out, a.v_out = _ptr(q_out), _ptr(k_out), _ptr(v_out)
    a.seq_len, a.d_model, a.n_heads, a.head_dim, a.eps = int(seq_len), int(d_model), int(n_heads), int(head_dim), float(eps)
    (a.stride_x_seq, a.stride_x_dim, a.stride_w_out, a.stride_w_in, a.stride_q_seq, a.stride_q_dim,
     a.stride_k_seq, a.stride_k_dim, a.stride_v_seq, a.stride_v_dim) = [int(s) for s in strides]
    a.dtype = _dtype_code(x)
    a.freqs_dtype = _dtype_code(freqs_cos)
    a.n_kv_heads = int(n_kv_heads)
    a.freqs_head_stride = int(freqs_head_stride)
    if freqs_strides is not None:
        a.stride_f_seq, a.stride_f_dim = [int(s) for s in freqs_strides]
    a.positions = _ptr(positions)
    check(lib().krt_fused_rmsnorm_qkv_rope(ctypes.byref(a), _stream(stream)))


def decode_workspace_bytes(num_tokens, d_model, n_heads, n_kv_heads, head_dim=128):
    return int(lib().krt_qkv_rope_decode_workspace_size(num_tokens, d_model, n_heads, n_kv_heads, head_dim))


def prefill_workspace_bytes(num_tokens, d_model, n_heads, n_kv_heads, head_dim=128):
    return int(lib().krt_qkv_rope_prefill_workspace_size(num_tokens, d_model, n_heads, n_kv_heads, head_dim))


def paged_args(x, qkv_weight, qkv_bias, rms_weight, rope_cos, rope_sin, positions, token_seq, block_table,
               kv_pool, q_out, n_heads, n_kv_heads, num_blocks, tokens_per_block, workspace, eps=1e-5,
               k_out=None, v_out=None, head_dim=128):
    a = QkvPagedArgs()
    a.x, a.qkv_weight, a.qkv_bias, a.rms_weight = _ptr(x), _ptr(qkv_weight), _ptr(qkv_bias), _ptr(rms_weight)
    a.rope_cos, a.rope_sin = _ptr(rope_cos), _ptr(rope_sin)
    a.positions, a.token_seq, a.block_table = _ptr(positions), _ptr(token_seq), _ptr(block_table)
    a.kv_pool, a.q_out, a.k_out, a.v_out = _ptr(kv_pool), _ptr(q_out), _ptr(k_out), _ptr(v_out)
    a.num_tokens, a.d_model = int(x.shape[0]), int(x.shape[1])
    a.n_heads, a.n_kv_heads, a.head_dim = int(n_heads), int(n_kv_heads), int(head_dim)
    a.x_stride, a.q_stride = int(x.stride(0)), int(q_out.stride(0))
    a.max_position = int(rope_cos.shape[0])
    a.num_seqs, a.block_table_stride = int(block_table.shape[0]), int(block_table.stride(0))
    a.num_blocks, a.tokens_per_block = int(num_blocks), int(tokens_per_block)
    a.eps = float(eps)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    a._refs = (x, qkv_weight, qkv_bias, rms_weight, rope_cos, rope_sin, positions, token_seq, block_table, kv_pool,
               q_out, k_out, v_out, workspace)
    return a


def qkv_rope_decode(args, stream=None):
    check(lib().krt_qkv_rope_decode(ctypes.byref(args), _stream(stream)))


def qkv_rope_prefill(args, stream=None):
    check(lib().krt_qkv_rope_prefill(ctypes.byref(args), _stream(stream)))


def read_status(workspace, stream=None):
    bits = _i32(0)
    rc = lib().krt_read_status(_ptr(workspace), _stream(stream), ctypes.byref(bits))
    return rc, bits.value


# ------------------------------------------------------------ communicator
def comm_create(rank, world_size, max_n_out):
    h = _vp()
    check(lib().krt_comm_create(int(rank), int(world_size), int(max_n_out), ctypes.byref(h)))
    return h


def comm_ipc_handle(comm):
    n = int(lib().krt_comm_handle_size())
    buf = ctypes.create_string_buffer(n)
    check(lib().krt_comm_ipc_handle(comm, buf))
    return buf.raw


def comm_open_peers(comm, handles):
    blob = b"".join(handles)
    check(lib().krt_comm_open_peers(comm, ctypes.c_char_p(blob)))


def nccl_unique_id():
    n = int(lib().krt_nccl_id_size())
    buf = ctypes.create_string_buffer(n)
    check(lib().krt_nccl_unique_id(buf))
    return buf.raw


def comm_attach_nccl(comm, nccl_id, threshold_bytes):
    check(lib().krt_comm_attach_nccl(comm, ctypes.c_char_p(nccl_id), ctypes.c_size_t(int(threshold_bytes))))


def comm_reset(comm, stream=None):
    check(lib().krt_comm_reset(comm, _stream(stream)))


def comm_destroy(comm):
    if comm:
        check(lib().krt_comm_destroy(comm))


def allreduce(comm, send, recv, status, stream=None):
    check(lib().krt_allreduce(comm, _ptr(send), _ptr(recv), int(send.numel()), _dtype_code(send), _ptr(status),
                              _stream(stream)))


def gemm_ar_workspace_bytes():
    return int(lib().krt_rowparallel_gemm_ar_workspace_size())


def gemm_ar_args(x, weight, y, workspace, residual=None):
    """residual: optional bf16 tensor with y's row stride (may be y itself):
    y = residual + allreduce(x @ weight^T)."""
    a = GemmArArgs()
    a.residual = _ptr(residual)
    a.x, a.weight, a.y = _ptr(x), _ptr(weight), _ptr(y)
    a.num_tokens, a.k_local = int(x.shape[0]), int(x.shape[1])
    a.n_out = int(weight.shape[0])
    a.x_stride, a.y_stride = int(x.stride(0)), int(y.stride(0))
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel() * workspace.element_size()
    a._refs = (x, weight, y, workspace, residual)
    return a


def rowparallel_gemm_ar(comm, args, stream=None):
    check(lib().krt_rowparallel_gemm_ar(comm, ctypes.byref(args), _stream(stream)))


# ------------------------------------------------------- paged attention
def attention_workspace_bytes(num_seqs, n_heads, n_kv_heads, max_seq_len):
    return int(lib().krt_paged_attention_workspace_size(num_seqs, n_heads, n_kv_heads, max_seq_len))


def attention_args(q, kv_pool, block_table, seq_lens, out, n_heads, n_kv_heads, num_blocks, tokens_per_block,
                   max_seq_len, workspace, scale=0.0, head_dim=128):
    """q / out: bf16 [num_seqs, >= n_heads * 128]; kv_pool: this layer's pool."""
    a = PagedAttentionArgs()
    a.q, a.kv_pool, a.block_table, a.seq_lens, a.out = (_ptr(q), _ptr(kv_pool), _ptr(block_table), _ptr(seq_lens),
                                                        _ptr(out))
    a.num_seqs, a.n_heads, a.n_kv_heads, a.head_dim = int(q.shape[0]), int(n_heads), int(n_kv_heads), int(head_dim)
    a.q_stride, a.out_stride = int(q.stride(0)), int(out.stride(0))
    a.block_table_stride, a.num_blocks = int(block_table.stride(0)), int(num_blocks)
    a.tokens_per_block, a.max_seq_len, a.scale = int(tokens_per_block), int(max_seq_len), float(scale)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel() * workspace.element_size()
    a._refs = (q, kv_pool, block_table, seq_lens, out, workspace)
    return a


def paged_attention_decode(args, stream=None):
    check(lib().krt_paged_attention_decode(ctypes.byref(args), _stream(stream)))


def prefill_attention_workspace_bytes():
    return int(lib().krt_paged_attention_prefill_workspace_size())


def prefill_attention_args(q, kv_pool, block_table, q_start, q_pos0, out, n_heads, n_kv_heads, num_blocks,
                           tokens_per_block, max_q_len, workspace, scale=0.0, head_dim=128):
    """q / out: bf16 [T, >= n_heads * 128] (sequence s's query rows q_start[s] ..
    q_start[s + 1] - 1); q_start int32 [num_seqs + 1]; q_pos0 int32 [num_seqs]."""
    a = PagedPrefillAttentionArgs()
    a.q, a.out, a.kv_pool, a.block_table = _ptr(q), _ptr(out), _ptr(kv_pool), _ptr(block_table)
    a.q_start, a.q_pos0 = _ptr(q_start), _ptr(q_pos0)
    a.num_seqs, a.n_heads, a.n_kv_heads, a.head_dim = int(q_pos0.shape[0]), int(n_heads), int(n_kv_heads), int(head_dim)
    a.q_stride, a.out_stride = int(q.stride(0)), int(out.stride(0))
    a.block_table_stride, a.num_blocks = int(block_table.stride(0)), int(num_blocks)
    a.tokens_per_block, a.max_q_len, a.scale = int(tokens_per_block), int(max_q_len), float(scale)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel() * workspace.element_size()
    a._refs = (q, kv_pool, block_table, q_start, q_pos0, out, workspace)
    return a


def paged_attention_prefill(args, stream=None):
    check(lib().krt_paged_attention_prefill(ctypes.byref(args), _stream(stream)))


# ------------------------------------------------- rest of the decode step
def projection_workspace_bytes(num_tokens, d_model):
    return int(lib().krt_projection_workspace_size(num_tokens, d_model))


def gate_up_args(x, rms_weight, gate_up_weight, act, workspace, eps=1e-5):
    """gate_up_weight: bf16 [2 * inter_local, d_model] in 64-row [gate | up] groups
    (interleave_gate_up)."""
    a = GateUpArgs()
    a.x, a.rms_weight, a.gate_up_weight, a.act = _ptr(x), _ptr(rms_weight), _ptr(gate_up_weight), _ptr(act)
    a.num_tokens, a.d_model = int(x.shape[0]), int(x.shape[1])
    a.inter_local = int(gate_up_weight.shape[0]) // 2
    a.x_stride, a.act_stride = int(x.stride(0)), int(act.stride(0))
    a.eps = float(eps)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel() * workspace.element_size()
    a._refs = (x, rms_weight, gate_up_weight, act, workspace)
    return a


def gate_up_swiglu(args, stream=None):
    check(lib().krt_gate_up_swiglu(ctypes.byref(args), _stream(stream)))


def interleave_gate_up(gate, up):
    """[inter, d] gate and up shards -> [2 * inter, d] in 64-row [gate | up] groups."""
    inter, d = gate.shape
    assert inter % 64 == 0 and up.shape == gate.shape
    return __import__("torch").stack([gate.view(inter // 64, 64, d), up.view(inter // 64, 64, d)], 1).reshape(
        2 * inter, d)


def lm_head_args(x, rms_weight, weight, keys, workspace, vocab_offset=0, eps=1e-5):
    a = LmHeadArgs()
    a.x, a.rms_weight, a.weight, a.argmax_keys = _ptr(x), _ptr(rms_weight), _ptr(weight), _ptr(keys)
    a.num_tokens, a.d_model = int(x.shape[0]), int(x.shape[1])
    a.vocab_local, a.vocab_offset = int(weight.shape[0]), int(vocab_offset)
    a.x_stride = int(x.stride(0))
    a.eps = float(eps)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel() * workspace.element_size()
    a._refs = (x, rms_weight, weight, keys, workspace)
    return a


def lm_head_argmax(args, stream=None):
    check(lib().krt_lm_head_argmax(ctypes.byref(args), _stream(stream)))


def greedy_step_args(keys, tokens, status, vocab, embedding=None, hidden=None, positions=None, seq_lens=None,
                     next_input=None):
    a = GreedyStepArgs()
    a.next_input = _ptr(next_input)
    a.argmax_keys, a.tokens, a.status = _ptr(keys), _ptr(tokens), _ptr(status)
    a.embedding, a.hidden, a.positions, a.seq_lens = _ptr(embedding), _ptr(hidden), _ptr(positions), _ptr(seq_lens)
    a.num_seqs = int(tokens.shape[0])
    a.d_model = 0 if embedding is None else int(embedding.shape[1])
    a.hidden_stride = 0 if hidden is None else int(hidden.stride(0))
    a.vocab = int(vocab)
    a._refs = (keys, tokens, status, embedding, hidden, positions, seq_lens, next_input)
    return a


def greedy_step(comm, args, stream=None):
    check(lib().krt_greedy_step(comm, ctypes.byref(args), _stream(stream)))


def argmax_key(value, index):
    """Host form of the (logit, index) key the kernels fold with atomicMax."""
    import struct
    u = struct.unpack("<I", struct.pack("<f", float(value)))[0]
    u = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - int(index))
