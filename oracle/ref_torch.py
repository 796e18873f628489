"""The reference's own torch decode path on the host CPU -- TEST INFRASTRUCTURE ONLY.

oracle/build_ref.py compiles the reference's python/lightdelta/reference package (post_conv_gdn,
reference/gdn.py:70-128), unmodified, to bytecode under oracle/_ref/torch_path/.  This module loads
it from there and runs it the way GDNBackend's packed "torch_reference" mode does
(python/lightdelta/backend.py:30-91):

  1. each request's initial state is the pool slot of its last accepted step,
     slots[r, accepted[r] - 1], zeroed when that step is invalid or the null slot (:40-44);
  2. the request's tokens cu[r] .. cu[r+1]-1 go through post_conv_gdn with lengths 0 for invalid
     requests and per-step checkpoints when the window is wider than one token (:48-73);
  3. every live step's output row is written, and its state is committed to its own slot (null
     destinations keep slot 0 unchanged) (:75-91).

The three steps are restated here rather than taken from backend.py because that module loads the
reference's operator library on import and hard-codes H=16, HV=48 (:57-61); this form takes the
head counts from the tensors, so it runs at the BASELINE geometry (H=16, HV=32).

Used by the tests (pinned against the C oracle) and by bench.py's CPU baselines, as the reference's
own CPU figure beside the C port; never by lightdelta_b200.
"""

from __future__ import annotations

import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BYTECODE_DIR = HERE / "_ref" / "torch_path"
# module name -> is a package, in load order (a module before the package that imports it)
MODULES = (("lightdelta", True), ("lightdelta.reference.gdn", False), ("lightdelta.reference", True))

_module = None


def available() -> bool:
    return all((BYTECODE_DIR / f"{name}.bytecode").exists() for name, _ in MODULES)


def reference():
    """The reference's lightdelta.reference package (GDNInputs, post_conv_gdn)."""
    global _module
    if _module is None:
        import importlib.machinery
        import importlib.util

        if not available():
            raise FileNotFoundError(f"{BYTECODE_DIR} holds no compiled reference: run python oracle/build_ref.py")
        loaded = sys.modules.get("lightdelta")
        if loaded is not None and getattr(loaded, "__file__", None) != str(BYTECODE_DIR / "lightdelta.bytecode"):
            raise RuntimeError(f"another lightdelta package is already imported ({loaded.__file__})")
        for name, package in MODULES:
            if name in sys.modules:
                continue
            loader = importlib.machinery.SourcelessFileLoader(name, str(BYTECODE_DIR / f"{name}.bytecode"))
            spec = importlib.util.spec_from_loader(name, loader, is_package=package)
            module = importlib.util.module_from_spec(spec)
            sys.modules[name] = module
            try:
                loader.exec_module(module)
            except BaseException:
                del sys.modules[name]
                raise
        _module = sys.modules["lightdelta.reference"]
    return _module


def packed_decode(qkv, a, b, a_log, dt_bias, slots, cu, accepted, pool, gate, weight, out, *, num_k_heads: int,
                  eps: float = 1e-6) -> None:
    """lightdelta::decode's contract on CPU torch tensors (bf16 activations, fp32 pool
    [slots, HV, V, K]): writes `out` rows and commits states into `pool` in place."""
    import torch

    ref = reference()
    batch, width = slots.shape
    value_heads, value_dim, key_dim = pool.shape[1:]
    steps = torch.arange(width)

    last = (accepted.clamp(1, width) - 1).long()
    source = slots.gather(1, last[:, None])[:, 0].long()
    valid = (accepted > 0) & (accepted <= width) & (source > 0)
    initial = pool.index_select(0, source.clamp_min(0))
    initial[~valid] = 0

    lengths = cu[1:] - cu[:-1]
    live = steps[None, :] < lengths[:, None]
    rows = (cu[:-1, None] + steps[None, :]).long()
    gathered = [x[rows.clamp(0, qkv.shape[0] - 1)] for x in (qkv, a, b, gate)]
    q, k, v = gathered[0].split((num_k_heads * key_dim, num_k_heads * key_dim, value_heads * value_dim), dim=-1)
    result = ref.post_conv_gdn(
        ref.GDNInputs(q.reshape(batch, width, num_k_heads, key_dim), k.reshape(batch, width, num_k_heads, key_dim),
                      v.reshape(batch, width, value_heads, value_dim), gathered[1], gathered[2], a_log, dt_bias,
                      gathered[3], weight),
        initial, torch.where(valid, lengths, 0), save_checkpoints=width > 1, norm_eps=eps)

    out.index_copy_(0, rows[live], result.output[live].reshape(-1, *out.shape[1:]))
    states = result.final_state[:, None] if width == 1 else result.checkpoints[:, 1:]
    commit = live & valid[:, None] & (slots > 0)
    pool.index_copy_(0, slots[commit].long(), states[commit])
