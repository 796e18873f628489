"""Device greedy MTP verification: the drop-in for LightDeltaRejectionSampler.

Mirrors python/lightdelta/runtime/speculation.py:271-326 (same class name, constructor and
call signature, same outputs) but runs as one ``torch.ops.lightdelta.greedy_verify`` launch:
no ``.tolist()``, no per-row host loop, no device round trip per comparison, so it can sit
inside a CUDA-graph-captured decode step.

Differences a caller can observe:
  * The reference raises ValueError when a request has more drafts than steps; this class
    raises the same error when ``num_draft_tokens_per_req`` is a host array (numpy / list, as
    vLLM passes it).  With device metadata the row is instead written as -1 / 0 / 0 and
    LD_FAULT_VERIFY_DRAFTS is set in the fault word, because raising would need a host sync.
  * Metadata that indexes outside the logits or input_ids (where the reference raises
    IndexError or wraps a negative index) gives -1 / 0 / 0 and LD_FAULT_VERIFY_RANGE.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops  # noqa: F401  (registers torch.ops.lightdelta.*; raises if the build is missing)


@dataclass
class SamplerOutput:
    """Field order of the SamplerOutput that speculation.py:326 constructs positionally."""

    sampled_token_ids: torch.Tensor
    logprobs_tensors: object | None
    num_nans: torch.Tensor | None
    num_sampled: torch.Tensor
    num_rejected: torch.Tensor


def _device_int32(values, count: int, device: torch.device) -> torch.Tensor:
    if isinstance(values, torch.Tensor):
        return values[:count].to(device=device, dtype=torch.int32, non_blocking=True).contiguous()
    host = torch.from_numpy(np.ascontiguousarray(np.asarray(values)[:count], dtype=np.int32))
    return host.to(device, non_blocking=True)


class LightDeltaRejectionSampler:
    """Greedy prefix verification for the fixed MTP service configuration."""

    def __init__(self, num_speculative_steps: int):
        self.num_speculative_steps = num_speculative_steps

    @torch.inference_mode()
    def __call__(self, logits, input_batch, draft_logits=None):
        if draft_logits is not None:
            raise ValueError("LightDelta greedy sampler does not accept draft logits")
        num_reqs = input_batch.num_reqs
        device = logits.device
        drafts = input_batch.num_draft_tokens_per_req
        if not isinstance(drafts, torch.Tensor):
            host = np.asarray(drafts)[:num_reqs]
            if host.size and int(host.max()) > self.num_speculative_steps:
                raise ValueError("invalid MTP draft-token metadata")
        token_dtype = input_batch.input_ids.dtype
        sampled = torch.empty((num_reqs, self.num_speculative_steps + 1), dtype=token_dtype, device=device)
        num_sampled = torch.empty(num_reqs, dtype=torch.int32, device=device)
        num_rejected = torch.empty_like(num_sampled)
        if num_reqs == 0:
            return SamplerOutput(sampled, None, None, num_sampled, num_rejected)
        torch.ops.lightdelta.greedy_verify(
            logits if logits.stride(-1) == 1 else logits.contiguous(),
            _device_int32(input_batch.cu_num_logits, num_reqs + 1, device),
            _device_int32(input_batch.query_start_loc, num_reqs + 1, device),
            input_batch.input_ids.to(device).contiguous(),
            _device_int32(drafts, num_reqs, device),
            _device_int32(input_batch.seq_lens, num_reqs, device),
            _device_int32(input_batch.prefill_len_np, num_reqs, device),
            sampled,
            num_sampled,
            num_rejected,
        )
        return SamplerOutput(sampled, None, None, num_sampled, num_rejected)
