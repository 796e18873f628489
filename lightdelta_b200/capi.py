"""ctypes binding of the C ABI in include/lightdelta_b200.h (liblightdelta_b200.so).

``lib()`` returns the raw CDLL with argument types set; the tensor helpers below call the
entry points with torch CUDA tensors (pointers, strides and the current stream), mirroring
the argument meaning of torch.ops.lightdelta.* without going through the dispatcher.
There is no CPU fallback: if the library is missing, loading raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblightdelta_b200.so"

LD_OK = 0
LD_ERR_INVALID = 1
LD_ERR_CUDA = 2
LD_DTYPE_F32 = 0
LD_DTYPE_BF16 = 1
LD_DTYPE_F16 = 2
LD_DTYPE_I32 = 3
LD_DTYPE_I64 = 4
LD_FAULT_DECODE_SLOT_RANGE = 0x1
LD_FAULT_DECODE_TOKENS = 0x2
LD_FAULT_GATHER_SLOT_RANGE = 0x4
LD_FAULT_SCATTER_SLOT_RANGE = 0x8
LD_FAULT_COPY_SLOT_RANGE = 0x10
LD_FAULT_WAIT_TIMEOUT = 0x20
LD_FAULT_VERIFY_DRAFTS = 0x40
LD_FAULT_VERIFY_RANGE = 0x80
LD_FAULT_CONV_SLOT_RANGE = 0x100
HEAD_DIM = 128
MAX_WIDTH = 4
MAX_VERIFY_STEPS = 7
DECODE_KERNELS = {"auto": 0, "rowreg": 1, "stream": 2}

_lib: ctypes.CDLL | None = None


class LightDeltaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `python -m lightdelta_b200.build` "
            "(lightdelta_b200 has no CPU fallback)"
        )
    handle = ctypes.CDLL(str(LIB_PATH))
    p, i64, i32, f32, u32p = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_uint32)
    handle.ld_last_error.argtypes = []
    handle.ld_last_error.restype = ctypes.c_char_p
    handle.ld_version.argtypes = []
    handle.ld_version.restype = ctypes.c_char_p
    handle.ld_decode.argtypes = [
        p, i64, p, i64, p, i64, p, p, i32, p, i64, i64, p, p, p, i64, i64, p, i64, p, i32, p, i64, i64, i64, f32, p,
    ]
    handle.ld_decode.restype = i32
    handle.ld_decode_bf16_state.argtypes = handle.ld_decode.argtypes
    handle.ld_decode_bf16_state.restype = i32
    handle.ld_gather_state.argtypes = [p, i64, i64, p, i64, p, i64, p, i64, i64, p]
    handle.ld_gather_state.restype = i32
    handle.ld_scatter_state.argtypes = [p, i64, p, i64, i64, p, i64, i64, i64, p]
    handle.ld_scatter_state.restype = i32
    handle.ld_copy_slots.argtypes = [p, i64, i64, p, i64, p, i64, i64, i64, p]
    handle.ld_copy_slots.restype = i32
    handle.ld_fault_flags.argtypes = [u32p, i32]
    handle.ld_fault_flags.restype = i32
    handle.ld_decode_kernel_override.argtypes = [i32]
    handle.ld_decode_kernel_override.restype = i32
    handle.ld_greedy_verify.argtypes = [p, i32, i64, i64, i64, p, p, p, i32, i64, p, p, p, i64, i64, p, p, p, p]
    handle.ld_greedy_verify.restype = i32
    handle.ld_greedy_verify_cluster_override.argtypes = [i32]
    handle.ld_greedy_verify_cluster_override.restype = i32
    handle.ld_conv_decode.argtypes = [
        p, i64, p, i64, p, i64, p, p, i32, p, i64, i64, p, p, p, i64, i64, p, i64, p, i32, p, i64, i64, i64, f32,
        p, i64, i64, i64, i64, i64, p, p, i64, p,
    ]
    handle.ld_conv_decode.restype = i32
    handle.ld_conv_update.argtypes = [p, i64, i64, i64, p, i64, i64, i64, i64, i64, p, p, i64, p, i64, p, p, i64, i64, p]
    handle.ld_conv_update.restype = i32
    handle.ld_programmatic_launch.argtypes = [i32]
    handle.ld_programmatic_launch.restype = i32
    handle.ld_decode_wait_test.argtypes = [i64, i32]
    handle.ld_decode_wait_test.restype = i32
    _lib = handle
    return handle


def last_error() -> str:
    return lib().ld_last_error().decode()


def version() -> str:
    return lib().ld_version().decode()


def check(rc: int) -> None:
    if rc != LD_OK:
        raise LightDeltaError(rc, last_error())


def fault_flags(clear: bool = True) -> int:
    """Device fault word of the current device (synchronises); see LD_FAULT_* constants."""
    value = ctypes.c_uint32(0)
    check(lib().ld_fault_flags(ctypes.byref(value), int(clear)))
    return value.value


def set_decode_kernel(name: str) -> str:
    """Select the kernel ld_decode launches (a key of DECODE_KERNELS); returns the previous
    selection.  All variants compute the same results."""
    previous = lib().ld_decode_kernel_override(DECODE_KERNELS[name])
    if previous < 0:
        raise LightDeltaError(-previous, last_error())
    return {v: k for k, v in DECODE_KERNELS.items()}[previous]


def set_decode_wait_test(limit_ns: int = 0, extra_tx_bytes: int = 0) -> None:
    """Bound of the persistent decode kernel's in-kernel waits (0: the default of one second) and
    the test-only over-count of each state load's expected bytes (0: off); see ld_decode_wait_test."""
    check(lib().ld_decode_wait_test(int(limit_ns), int(extra_tx_bytes)))


def set_programmatic_launch(enable: bool) -> bool:
    """Enable or disable programmatic dependent launch for every kernel; returns the previous
    setting.  Results do not depend on it."""
    return bool(lib().ld_programmatic_launch(1 if enable else 0))


def set_verify_cluster(cluster: int) -> int:
    """Force ld_greedy_verify's cluster size (1, 2, 4 or 8 CTAs per request; 0 = automatic);
    returns the previous setting.  Results do not depend on it."""
    previous = lib().ld_greedy_verify_cluster_override(int(cluster))
    if previous < 0:
        raise LightDeltaError(-previous, last_error())
    return previous


# ---------------------------------------------------------------------------------------------
# torch-tensor helpers (C-ABI path)
# ---------------------------------------------------------------------------------------------
def _stream(tensor, stream) -> int:
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(tensor.device)
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _dtype_code(tensor) -> int:
    import torch

    if tensor.dtype == torch.bfloat16:
        return LD_DTYPE_BF16
    if tensor.dtype == torch.float32:
        return LD_DTYPE_F32
    raise TypeError(f"unsupported dtype {tensor.dtype}")


def decode(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out, eps=1e-6, stream=None):
    """ld_decode on torch tensors laid out as torch.ops.lightdelta.decode expects; a bf16 `state`
    pool goes to ld_decode_bf16_state."""
    import torch

    hv = state.shape[1]
    h = (qkv.shape[1] // HEAD_DIM - hv) // 2
    entry = lib().ld_decode_bf16_state if state.dtype == torch.bfloat16 else lib().ld_decode
    check(entry(
        qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a_log.data_ptr(),
        dt_bias.data_ptr(), _dtype_code(dt_bias), indices.data_ptr(), indices.shape[0], indices.shape[1],
        cu.data_ptr(), accepted.data_ptr(), state.data_ptr(), state.shape[0], state.stride(0), gate.data_ptr(),
        gate.stride(0), weight.data_ptr(), _dtype_code(weight), out.data_ptr(), qkv.shape[0], h, hv, float(eps),
        _stream(qkv, stream),
    ))


def _slot_elems(pool) -> int:
    n = 1
    for d in pool.shape[1:]:
        n *= d
    return n


def gather_state(pool, slots, valid, out, stream=None):
    check(lib().ld_gather_state(
        pool.data_ptr(), pool.shape[0], pool.stride(0), slots.data_ptr(), slots.stride(0), valid.data_ptr(),
        slots.numel(), out.data_ptr(), out.stride(0), _slot_elems(pool), _stream(pool, stream),
    ))


def scatter_state(packed, slots, pool, stream=None):
    check(lib().ld_scatter_state(
        packed.data_ptr(), packed.stride(0), slots.data_ptr(), slots.stride(0), slots.numel(), pool.data_ptr(),
        pool.shape[0], pool.stride(0), _slot_elems(pool), _stream(pool, stream),
    ))


def copy_slots(pool, src, dst, stream=None):
    check(lib().ld_copy_slots(
        pool.data_ptr(), pool.shape[0], pool.stride(0), src.data_ptr(), src.stride(0), dst.data_ptr(),
        dst.stride(0), src.numel(), _slot_elems(pool), _stream(pool, stream),
    ))


def greedy_verify(logits, cu_num_logits, query_start_loc, input_ids, num_draft_tokens, seq_lens, prefill_len,
                  sampled, num_sampled, num_rejected, stream=None):
    """ld_greedy_verify on torch tensors laid out as torch.ops.lightdelta.greedy_verify expects."""
    import torch

    logits_code = {torch.float32: LD_DTYPE_F32, torch.bfloat16: LD_DTYPE_BF16, torch.float16: LD_DTYPE_F16}
    token_code = {torch.int32: LD_DTYPE_I32, torch.int64: LD_DTYPE_I64}
    check(lib().ld_greedy_verify(
        logits.data_ptr(), logits_code[logits.dtype], logits.shape[0], logits.shape[1], logits.stride(0),
        cu_num_logits.data_ptr(), query_start_loc.data_ptr(), input_ids.data_ptr(), token_code[input_ids.dtype],
        input_ids.numel(), num_draft_tokens.data_ptr(), seq_lens.data_ptr(), prefill_len.data_ptr(),
        num_draft_tokens.numel(), sampled.shape[1] - 1, sampled.data_ptr(), num_sampled.data_ptr(),
        num_rejected.data_ptr(), _stream(logits, stream),
    ))


def conv_decode(qkv, conv_state, conv_weight, conv_bias, a, b, a_log, dt_bias, indices, cu, accepted, state, gate,
                weight, out, eps=1e-6, stream=None):
    """ld_conv_decode on torch tensors laid out as torch.ops.lightdelta.conv_decode expects."""
    hv = state.shape[1]
    h = (qkv.shape[1] // HEAD_DIM - hv) // 2
    w = conv_weight.reshape(conv_weight.shape[0], -1)
    check(lib().ld_conv_decode(
        qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a_log.data_ptr(),
        dt_bias.data_ptr(), _dtype_code(dt_bias), indices.data_ptr(), indices.shape[0], indices.shape[1],
        cu.data_ptr(), accepted.data_ptr(), state.data_ptr(), state.shape[0], state.stride(0), gate.data_ptr(),
        gate.stride(0), weight.data_ptr(), _dtype_code(weight), out.data_ptr(), qkv.shape[0], h, hv, float(eps),
        conv_state.data_ptr(), conv_state.shape[0], conv_state.stride(0), conv_state.stride(1), conv_state.stride(2),
        conv_state.shape[2], w.data_ptr(), None if conv_bias is None else conv_bias.data_ptr(), w.shape[1],
        _stream(qkv, stream),
    ))


def conv_update(x, conv_state, conv_weight, conv_bias, slots, accepted, cu, max_tokens, stream=None):
    """ld_conv_update on torch tensors laid out as torch.ops.lightdelta.conv_update expects."""
    w = conv_weight.reshape(conv_weight.shape[0], -1)
    check(lib().ld_conv_update(
        x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], conv_state.data_ptr(), conv_state.shape[0],
        conv_state.stride(0), conv_state.stride(1), conv_state.stride(2), conv_state.shape[2], w.data_ptr(),
        None if conv_bias is None else conv_bias.data_ptr(), w.shape[1], slots.data_ptr(), slots.stride(0),
        None if accepted is None else accepted.data_ptr(), cu.data_ptr(), slots.numel(), int(max_tokens),
        _stream(x, stream),
    ))


def decode_packed_noalloc(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out, eps=1e-6,
                          stream=None):
    """ld_decode_packed_noalloc on torch tensors laid out as torch.ops.lightdelta.decode expects:
    the packed state path with its scratch in the library's static device array (fp32 pool only;
    at most LD_NOALLOC_SCRATCH_BYTES of scratch, see include/lightdelta_b200.h)."""
    handle = lib()
    entry = handle.ld_decode_packed_noalloc
    if entry.argtypes is None:
        entry.argtypes = handle.ld_decode.argtypes
        entry.restype = ctypes.c_int
    hv = state.shape[1]
    h = (qkv.shape[1] // HEAD_DIM - hv) // 2
    check(entry(
        qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a_log.data_ptr(),
        dt_bias.data_ptr(), _dtype_code(dt_bias), indices.data_ptr(), indices.shape[0], indices.shape[1],
        cu.data_ptr(), accepted.data_ptr(), state.data_ptr(), state.shape[0], state.stride(0), gate.data_ptr(),
        gate.stride(0), weight.data_ptr(), _dtype_code(weight), out.data_ptr(), qkv.shape[0], h, hv, float(eps),
        _stream(qkv, stream),
    ))
