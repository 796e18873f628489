"""The reference's own decode kernel at any value-head ratio -- TEST INFRASTRUCTURE ONLY.

Loads oracle/_ref/libref_harness.so (built by oracle/build_ref.py from the reference's unmodified
csrc/gdn_decode.cu) and launches gdn_decode_post_conv_mtp_kernel<float, ratio, false>
(csrc/gdn_decode.cu:130-354) with the stock launcher's grid, block and arguments
(csrc/gdn_decode.cu:407-418), for ratio 2 (the BASELINE geometry H=16, HV=32) or 3.  Used by the
GPU tests as a comparison kernel and by bench.py's reference arm; never by lightdelta_b200.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
HARNESS = HERE / "_ref" / "libref_harness.so"
HEAD_DIM = 128

_lib = None


def available() -> bool:
    return HARNESS.exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not HARNESS.exists():
            raise FileNotFoundError(f"{HARNESS} is missing: build it with python oracle/build_ref.py")
        handle = ctypes.CDLL(str(HARNESS))
        p, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        handle.ref_decode_launch.argtypes = [p, i64, p, i64, p, i64, p, p, i32, p, i32, i32, p, p, p, i64, p, i64, p,
                                             i32, p, i32, i32, f32, p]
        handle.ref_decode_launch.restype = i32
        _lib = handle
    return _lib


def decode(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out, eps=1e-6, stream=None):
    """One launch of the reference kernel on torch CUDA tensors laid out as lightdelta::decode
    expects (fp32 pool; H and HV taken from the tensors)."""
    import torch

    hv = state.shape[1]
    h = (qkv.shape[1] // HEAD_DIM - hv) // 2
    if stream is None:
        stream = torch.cuda.current_stream(qkv.device)
    rc = lib().ref_decode_launch(
        qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a_log.data_ptr(),
        dt_bias.data_ptr(), int(dt_bias.dtype == torch.bfloat16), indices.data_ptr(), indices.shape[0],
        indices.shape[1], cu.data_ptr(), accepted.data_ptr(), state.data_ptr(), state.stride(0), gate.data_ptr(),
        gate.stride(0), weight.data_ptr(), int(weight.dtype == torch.bfloat16), out.data_ptr(), h, hv, float(eps),
        stream.cuda_stream)
    if rc != 0:
        raise RuntimeError(f"reference kernel launch failed ({rc})")
