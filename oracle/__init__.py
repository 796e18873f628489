"""CPU oracle for the lightdelta_b200 hot path -- TEST INFRASTRUCTURE ONLY.

The parity checker of tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py.
Nothing in lightdelta_b200/ imports or calls this package.

It wraps oracle/gdn_oracle.c (built by oracle/Makefile into oracle/_build/) with numpy
entry points.  bf16 tensors travel as numpy uint16 arrays holding the raw bf16 bits.

Functions and the reference code they restate:
  post_conv_gdn      python/lightdelta/reference/gdn.py:70-128
  decode             csrc/gdn_decode.cu:130-354 contract (python/lightdelta/backend.py:24-91)
  gather_state       csrc/state_io.cu:11-27, :44-58
  scatter_state      csrc/state_io.cu:11-27, :60-69
  copy_slots         python/lightdelta/backend.py:87-91 for states already in the pool
  greedy_verify      python/lightdelta/runtime/speculation.py:274-326 (oracle/greedy_oracle.c)
  conv_update        vLLM causal_conv1d_update as python/lightdelta/integration/vllm_layer.py:161-172
                     and :199-207 call it (oracle/conv_oracle.c)
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libgdn_oracle.so"
HEAD_DIM = 128

_lib = None


def build(force: bool = False) -> Path:
    """Compile the C restatement (make), if missing or stale."""
    stale = (
        force
        or not LIB_PATH.exists()
        or any(p.stat().st_mtime > LIB_PATH.stat().st_mtime for p in (HERE / "gdn_oracle.c", HERE / "greedy_oracle.c", HERE / "conv_oracle.c",
                                                               HERE / "Makefile"))
    )
    if stale:
        subprocess.run(["make", "-s", "-C", str(HERE)] + (["-B"] if force else []), check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        handle = ctypes.CDLL(str(LIB_PATH))
        p, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        handle.oracle_post_conv_gdn.argtypes = [i64] * 6 + [p] * 11 + [i32, f32, p, p, p, i32]
        handle.oracle_post_conv_gdn.restype = i32
        handle.oracle_decode_state.argtypes = [
            p, i64, p, i64, p, i64, p, p, i32, p, i64, i64, p, p, p, i32, i64, i64, p, i64, p, i32, p, i64, i64,
            i64, f32, i32,
        ]
        handle.oracle_decode_state.restype = i32
        handle.oracle_gather_state.argtypes = [p, i64, i64, p, i64, p, i64, p, i64, i64, i32]
        handle.oracle_gather_state.restype = None
        handle.oracle_scatter_state.argtypes = [p, i64, p, i64, i64, p, i64, i64, i64]
        handle.oracle_scatter_state.restype = None
        handle.oracle_copy_slots.argtypes = [p, i64, i64, p, i64, p, i64, i64, i64]
        handle.oracle_copy_slots.restype = None
        handle.oracle_argmax_rows.argtypes = [p, i32, i64, i64, i64, p, i32]
        handle.oracle_argmax_rows.restype = None
        handle.oracle_greedy_verify.argtypes = [p, i32, i64, i64, i64, p, p, p, i64, p, p, p, i64, i64, p, p, p, p, i32]
        handle.oracle_greedy_verify.restype = ctypes.c_uint32
        handle.oracle_conv_update.argtypes = [p, i64, p, i64, p, i32, i64, i64, i64, i64, i64, p, i32, p, i64, i64,
                                              p, i64, p, p, i64, i64]
        handle.oracle_conv_update.restype = i32
        _lib = handle
    return _lib


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def _ptr(array: np.ndarray | None) -> int | None:
    return None if array is None else array.ctypes.data


def _dense(array, dtype) -> np.ndarray:
    out = np.ascontiguousarray(array, dtype=dtype)
    return out


# ---------------------------------------------------------------------------------------------
# bf16 helpers (round to nearest even, as torch and CUDA __float2bfloat16_rn)
# ---------------------------------------------------------------------------------------------
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)


# ---------------------------------------------------------------------------------------------
# post_conv_gdn (gdn.py:70-128)
# ---------------------------------------------------------------------------------------------
def post_conv_gdn(q, k, v, a, b, a_log, dt_bias, gate, norm_weight, initial_state, lengths, *,
                  io_bf16: bool, save_checkpoints: bool = False, norm_eps: float = 1e-6, threads: int = 0):
    """fp32 numpy arrays in the reference's shapes; returns (output, final_state, checkpoints|None)."""
    q, k, v = (_dense(x, np.float32) for x in (q, k, v))
    B, T, Hk, K = q.shape
    Hv, V = v.shape[2], v.shape[3]
    a, b, gate = (_dense(x, np.float32) for x in (a, b, gate))
    a_log, dt_bias, norm_weight = (_dense(x, np.float32) for x in (a_log, dt_bias, norm_weight))
    initial_state = _dense(initial_state, np.float32)
    lengths = _dense(lengths, np.int64)
    assert initial_state.shape == (B, Hv, V, K)
    output = np.empty((B, T, Hv, V), np.float32)
    final = np.empty((B, Hv, V, K), np.float32)
    checkpoints = np.empty((B, T + 1, Hv, V, K), np.float32) if save_checkpoints else None
    rc = lib().oracle_post_conv_gdn(
        B, T, Hk, Hv, K, V, _ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(a_log), _ptr(dt_bias), _ptr(gate),
        _ptr(norm_weight), _ptr(initial_state), _ptr(lengths), int(io_bf16), norm_eps, _ptr(output), _ptr(final),
        _ptr(checkpoints), threads,
    )
    if rc != 0:
        raise ValueError("oracle_post_conv_gdn: invalid geometry")
    return output, final, checkpoints


# ---------------------------------------------------------------------------------------------
# pool-indexed decode / verify (gdn_decode.cu:130-354 contract)
# ---------------------------------------------------------------------------------------------
def decode(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out, *, num_k_heads: int,
           eps: float = 1e-6, threads: int = 0) -> None:
    """In-place on `state` ([S,HV,128,128]) and `out` (uint16 [N,HV,128]).

    qkv, a, b, gate, out are uint16 (bf16 bits) 2-D/3-D arrays whose last dimension is dense
    (row strides may exceed the row); dt_bias and weight may be float32 or uint16 (bf16).
    `state` is float32 (the reference's pool) or uint16 bf16 bits (a bf16 pool: fp32 recurrence,
    each stored step rounded to bf16).
    """
    for name, arr in (("qkv", qkv), ("a", a), ("b", b), ("gate", gate), ("out", out)):
        if arr.dtype != np.uint16 or arr.strides[-1] != 2:
            raise TypeError(f"{name} must be a uint16 (bf16 bits) array with a dense last dimension")
    if state.dtype not in (np.float32, np.uint16) or not state[0].flags.c_contiguous:
        raise TypeError("state must be float32 or uint16 (bf16 bits) with dense slots")
    if gate.ndim != 3 or gate.strides[1] != HEAD_DIM * 2 or not out.flags.c_contiguous:
        raise TypeError("gate must be [N,HV,128] with head stride 128 and out contiguous")
    indices = _dense(indices, np.int32)
    cu = _dense(cu, np.int32)
    accepted = _dense(accepted, np.int32)
    a_log = _dense(a_log, np.float32)
    dt_bias_bf16 = dt_bias.dtype == np.uint16
    weight_bf16 = weight.dtype == np.uint16
    dt_bias = _dense(dt_bias, np.uint16 if dt_bias_bf16 else np.float32)
    weight = _dense(weight, np.uint16 if weight_bf16 else np.float32)
    R, W = indices.shape
    S, HV = state.shape[0], state.shape[1]
    rc = lib().oracle_decode_state(
        _ptr(qkv), qkv.strides[0] // 2, _ptr(a), a.strides[0] // 2, _ptr(b), b.strides[0] // 2, _ptr(a_log),
        _ptr(dt_bias), int(dt_bias_bf16), _ptr(indices), R, W, _ptr(cu), _ptr(accepted), _ptr(state),
        int(state.dtype == np.uint16), S, state.strides[0] // state.itemsize, _ptr(gate), gate.strides[0] // 2, _ptr(weight), int(weight_bf16), _ptr(out),
        qkv.shape[0], num_k_heads, HV, eps, threads,
    )
    if rc != 0:
        raise ValueError("oracle_decode: invalid arguments")


# ---------------------------------------------------------------------------------------------
# state-pool copies (state_io.cu:11-69)
# ---------------------------------------------------------------------------------------------
def _slot_view(pool: np.ndarray) -> tuple[int, int]:
    if pool.dtype != np.float32 or not pool[0].flags.c_contiguous:
        raise TypeError("pool rows must be float32 with dense inner dimensions")
    return pool.strides[0] // 4, int(np.prod(pool.shape[1:]))


def _vector(slots: np.ndarray) -> tuple[np.ndarray, int]:
    if slots.dtype != np.int32 or slots.ndim != 1:
        raise TypeError("slots must be an int32 vector")
    return slots, slots.strides[0] // 4


def gather_state(pool: np.ndarray, slots: np.ndarray, valid: np.ndarray, out: np.ndarray, threads: int = 0) -> None:
    pool_stride, elems = _slot_view(pool)
    out_stride, _ = _slot_view(out)
    slots, slots_stride = _vector(slots)
    valid = _dense(valid, np.uint8)
    lib().oracle_gather_state(_ptr(pool), pool.shape[0], pool_stride, _ptr(slots), slots_stride, _ptr(valid),
                              slots.shape[0], _ptr(out), out_stride, elems, threads)


def scatter_state(packed: np.ndarray, slots: np.ndarray, pool: np.ndarray) -> None:
    pool_stride, elems = _slot_view(pool)
    packed_stride, _ = _slot_view(packed)
    slots, slots_stride = _vector(slots)
    lib().oracle_scatter_state(_ptr(packed), packed_stride, _ptr(slots), slots_stride, slots.shape[0], _ptr(pool),
                               pool.shape[0], pool_stride, elems)


def copy_slots(pool: np.ndarray, src: np.ndarray, dst: np.ndarray) -> None:
    pool_stride, elems = _slot_view(pool)
    src, src_stride = _vector(src)
    dst, dst_stride = _vector(dst)
    lib().oracle_copy_slots(_ptr(pool), pool.shape[0], pool_stride, _ptr(src), src_stride, _ptr(dst), dst_stride,
                            src.shape[0], elems)


# ---------------------------------------------------------------------------------------------
# greedy MTP verification (speculation.py:274-326)
# ---------------------------------------------------------------------------------------------
VERIFY_FAULT_DRAFTS = 0x40
VERIFY_FAULT_RANGE = 0x80


def _logits_view(logits: np.ndarray) -> tuple[np.ndarray, int, int]:
    """(array, dtype code, row stride in elements); bf16 / f16 travel as uint16 bits."""
    if logits.ndim != 2 or logits.strides[1] != logits.itemsize:
        raise TypeError("logits must be a matrix with a dense last dimension")
    if logits.dtype == np.float32:
        code = 0
    elif logits.dtype == np.uint16:
        code = 1  # bf16 bits
    elif logits.dtype == np.float16:
        code = 2
    else:
        raise TypeError(f"unsupported logits dtype {logits.dtype}")
    return logits, code, logits.strides[0] // logits.itemsize


def argmax_rows(logits: np.ndarray, threads: int = 0) -> np.ndarray:
    """torch.argmax(logits, -1) for float32, float16 or bf16-bits (uint16) rows."""
    logits, code, stride = _logits_view(logits)
    target = np.empty(logits.shape[0], np.int64)
    lib().oracle_argmax_rows(_ptr(logits), code, logits.shape[0], logits.shape[1], stride, _ptr(target), threads)
    return target


def greedy_verify(logits, cu_num_logits, query_start_loc, input_ids, num_draft_tokens, seq_lens, prefill_len,
                  num_speculative_steps: int, threads: int = 0):
    """Returns (sampled int64 [R, steps+1], num_sampled int32 [R], num_rejected int32 [R], faults)."""
    logits, code, stride = _logits_view(logits)
    cu_num_logits, query_start_loc, num_draft_tokens, seq_lens, prefill_len = (
        _dense(x, np.int32) for x in (cu_num_logits, query_start_loc, num_draft_tokens, seq_lens, prefill_len))
    input_ids = _dense(input_ids, np.int64)
    n = num_draft_tokens.shape[0]
    sampled = np.empty((n, num_speculative_steps + 1), np.int64)
    num_sampled = np.empty(n, np.int32)
    num_rejected = np.empty(n, np.int32)
    target = np.empty(max(1, logits.shape[0]), np.int64)
    faults = lib().oracle_greedy_verify(
        _ptr(logits), code, logits.shape[0], logits.shape[1], stride, _ptr(cu_num_logits), _ptr(query_start_loc),
        _ptr(input_ids), input_ids.shape[0], _ptr(num_draft_tokens), _ptr(seq_lens), _ptr(prefill_len), n,
        num_speculative_steps, _ptr(sampled), _ptr(num_sampled), _ptr(num_rejected), _ptr(target), threads,
    )
    return sampled, num_sampled, num_rejected, int(faults)


# ---------------------------------------------------------------------------------------------
# causal conv1d state update (vLLM causal_conv1d_update, vllm_layer.py:161-172, :199-207)
# ---------------------------------------------------------------------------------------------
def _elem_code(array: np.ndarray) -> int:
    if array.dtype == np.float32:
        return 0
    if array.dtype == np.uint16:
        return 1  # bf16 bits
    raise TypeError(f"unsupported dtype {array.dtype}")


def conv_update(x, state, weight, bias, slots, accepted, query_start_loc) -> np.ndarray:
    """Updates `state` ([slots, dim, L] view, any strides) in place and returns the post-conv
    activations (same dtype as x / state: float32, or uint16 bf16 bits)."""
    if x.dtype != state.dtype or x.ndim != 2 or x.strides[1] != x.itemsize:
        raise TypeError("x must be a matrix of the state dtype with a dense last dimension")
    if state.ndim != 3:
        raise TypeError("state must be [slots, dim, L]")
    weight = np.ascontiguousarray(weight)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=weight.dtype)
    slots, slots_stride = np.ascontiguousarray(slots, dtype=np.int32), 1
    accepted = _dense(accepted, np.int32)
    query_start_loc = _dense(query_start_loc, np.int32)
    y = np.empty(x.shape, x.dtype)
    item = state.itemsize
    rc = lib().oracle_conv_update(
        _ptr(x), x.strides[0] // x.itemsize, _ptr(y), y.shape[1], _ptr(state), _elem_code(state), state.shape[0],
        state.strides[0] // item, state.strides[1] // item, state.strides[2] // item, state.shape[2], _ptr(weight),
        _elem_code(weight), _ptr(bias), weight.shape[0], weight.shape[1], _ptr(slots), slots_stride,
        _ptr(accepted), _ptr(query_start_loc), slots.shape[0], x.shape[0],
    )
    if rc != 0:
        raise ValueError("oracle_conv_update: invalid arguments")
    return y
