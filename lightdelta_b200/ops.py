"""torch.library registration of the ``lightdelta`` operators.

Mirror of the reference's python/lightdelta/ops/__init__.py:1-21: importing this module loads
the native registration library (here lightdelta_b200/_C.so, built for sm_100a) and registers
no-op fake kernels so the ops can be traced.  After import, ``torch.ops.lightdelta.decode``,
``gather_state`` and ``scatter_state`` have the reference's exact schemas; ``copy_state`` is an
extension.  A missing library raises: there is no CPU fallback.
"""

from __future__ import annotations

from pathlib import Path

import torch

from lightdelta_b200 import capi

LIB_PATH = Path(__file__).resolve().parent / "_C.so"

if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is missing; build it with `python -m lightdelta_b200.build`")
capi.lib()  # the C-ABI library must be loadable too (it is _C.so's dependency)
torch.ops.load_library(str(LIB_PATH))


@torch.library.register_fake("lightdelta::decode")
def _decode_fake(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out, eps):
    return None


@torch.library.register_fake("lightdelta::decode_bf16_state")
def _decode_bf16_state_fake(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out, eps):
    return None


@torch.library.register_fake("lightdelta::gather_state")
def _gather_fake(pool, slots, valid, out):
    return None


@torch.library.register_fake("lightdelta::scatter_state")
def _scatter_fake(packed, slots, pool):
    return None


@torch.library.register_fake("lightdelta::copy_state")
def _copy_fake(pool, src, dst):
    return None


@torch.library.register_fake("lightdelta::greedy_verify")
def _greedy_verify_fake(logits, cu_num_logits, query_start_loc, input_ids, num_draft_tokens, seq_lens, prefill_len,
                        sampled, num_sampled, num_rejected):
    return None


@torch.library.register_fake("lightdelta::conv_decode")
def _conv_decode_fake(qkv, conv_state, conv_weight, conv_bias, a, b, a_log, dt_bias, indices, cu, accepted, state,
                      gate, weight, out, eps):
    return None


@torch.library.register_fake("lightdelta::conv_update")
def _conv_update_fake(x, conv_state, conv_weight, conv_bias, slots, accepted, cu, max_tokens):
    return None
