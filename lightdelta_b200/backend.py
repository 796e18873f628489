"""The post-convolution GDN boundary: mirror of python/lightdelta/backend.py:11-91.

``GDNBackend(config)(qkv, a, b, a_log, dt_bias, slots, cu, accepted, pool, gate, weight, out, eps)``
has the reference's call signature and state semantics:

* ``state_io = "indexed"`` (backend.py:24-28): one ``lightdelta::decode`` directly on the pool.
  The source state is ``slots[r, accepted[r]-1]``; step t's state lands in ``slots[r, t]``, so an
  MTP commit is the next step's choice of source slot (no copy).
* ``state_io = "packed"`` (backend.py:30-91): gather each request's source state into a scratch
  buffer (``lightdelta::gather_state``: invalid requests get a zero state), decode on the scratch,
  then commit every live step state to its slot (``lightdelta::scatter_state``; null destination
  slots are skipped, which leaves slot 0 untouched exactly as the reference's index_copy_ of
  pool[0] onto itself does).

Only ``compute = "cuda_fused"`` exists here: the reference's Torch compute mode is this
project's parity oracle and is not offered as a product path.  The config may be this package's
``BackendConfig`` or the reference's own (``python/lightdelta/config.py``): the backend calls its
``validate()`` and reads only ``compute`` and ``state_io``.

A bf16 pool (an extension; the reference's pool is fp32) runs in indexed mode through
``lightdelta::decode_bf16_state``.  Packed mode keeps the reference's fp32-only state copies.
"""

from __future__ import annotations

from collections import Counter

import torch

from lightdelta_b200 import ops  # noqa: F401 -- registers torch.ops.lightdelta


class GDNBackend:
    def __init__(self, config):
        config.validate()
        if getattr(config, "compute", None) != "cuda_fused":
            raise ValueError(
                "lightdelta_b200 implements compute='cuda_fused' only; the Torch reference compute "
                "mode is the parity oracle, not a backend"
            )
        if getattr(config, "state_io", None) not in ("packed", "indexed"):
            raise ValueError("state_io must be packed or indexed")
        self.config = config
        self.calls = Counter()
        self._packed: dict = {}

    def __call__(self, qkv, a, b, a_log, dt_bias, slots, cu, accepted, pool, gate, weight, out, eps=1e-6):
        batch, width = slots.shape
        self.calls["decode" if width == 1 else "verify"] += 1
        if self.config.state_io == "indexed":
            op = torch.ops.lightdelta.decode_bf16_state if pool.dtype == torch.bfloat16 else torch.ops.lightdelta.decode
            op(qkv, a, b, a_log, dt_bias, slots, cu, accepted, pool, gate, weight, out, eps)
            return
        if pool.dtype != torch.float32:
            raise ValueError("packed state I/O needs an fp32 pool (gather_state and scatter_state copy fp32 slots); "
                             "use state_io='indexed' for a bf16 pool")

        key = (pool.device, batch, width, tuple(pool.shape[1:]))
        if key not in self._packed:
            scratch = pool.new_empty((1 + batch * width, *pool.shape[1:]))
            compact = torch.arange(1, 1 + batch * width, device=pool.device, dtype=torch.int32).view(batch, width)
            ones = torch.ones(batch, device=pool.device, dtype=torch.int32)
            offsets = torch.arange(width, device=pool.device, dtype=torch.int32)[None, :]
            self._packed[key] = scratch, compact, ones, offsets
        scratch, compact, ones, offsets = self._packed[key]
        source = slots.gather(1, (accepted.clamp(1, width) - 1)[:, None].long()).flatten()
        valid = (accepted > 0) & (accepted <= width) & (source > 0)
        initial = scratch[1:].view(batch, width, *pool.shape[1:])[:, 0]
        torch.ops.lightdelta.gather_state(pool, source, valid, initial)
        indices = torch.where(valid[:, None], compact, 0)
        torch.ops.lightdelta.decode(qkv, a, b, a_log, dt_bias, indices, cu, ones, scratch, gate, weight, out, eps)
        lengths = cu[1:] - cu[:-1]
        live = offsets < lengths[:, None]
        destinations = torch.where(live & valid[:, None] & (slots > 0), slots, 0).flatten()
        torch.ops.lightdelta.scatter_state(scratch[1:], destinations, pool)
