"""Seeded synthetic workloads with the shapes and distributions of the BASELINE configs.

No public dataset exists for this path; these builders restate the configurations:
  config 1  decode, B=1, T=1                           (CPU-runnable reference case)
  config 2  indexed decode, B=256, T=1, pool of 1024 fp32 slots [32,128,128]
  config 3  MTP verify, B=64, T=4, accepted ~ U{1..4}, distinct slots per (request, step)
  config 4  state-pool copy, pools of 2048 slots, gather 512 slots then scatter to a permutation
  config 5  stacked decode over 48 layers (T=4 verify), state sharded by sequence slot
  sampling  config 3's greedy draft verification: 64 requests x 3 drafts, 4 logits rows each over
            a 151,936-token (Qwen3) vocabulary, accepted drafts ~ U{0..3}
Geometry: H=16 key heads, HV=32 value heads (ratio 2), K=V=128.  q, k, v ~ N(0,1) bf16; a_log =
dt_bias = 0 so g = -softplus(a) with a ~ N(0,1); b ~ N(0,1) (beta = sigmoid(b)); gate 0.2*N(0,1);
norm weight N(0,1) bf16; state fp32 N(0, 0.02^2).  qkv and gate are slices of one wider
projection buffer and a, b slices of another, as vLLM lays them out (reference
tests/conftest.py:14-28).  Slot 0 is the reserved null slot and is never selected.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

HEAD_DIM = 128
SLOT_HEAD_BYTES = HEAD_DIM * HEAD_DIM * 4


@dataclass
class DecodeCase:
    """Arguments of one lightdelta::decode call plus bookkeeping for byte accounting."""

    qkv: torch.Tensor
    a: torch.Tensor
    b: torch.Tensor
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    slots: torch.Tensor
    cu: torch.Tensor
    accepted: torch.Tensor
    pool: torch.Tensor
    gate: torch.Tensor
    weight: torch.Tensor
    out: torch.Tensor
    eps: float = 1e-6
    num_k_heads: int = 16
    extra: dict = field(default_factory=dict)

    def kwargs(self) -> dict:
        return dict(qkv=self.qkv, a=self.a, b=self.b, a_log=self.a_log, dt_bias=self.dt_bias, slots=self.slots,
                    cu=self.cu, accepted=self.accepted, pool=self.pool, gate=self.gate, weight=self.weight,
                    out=self.out, eps=self.eps)

    def op_args(self) -> tuple:
        """Positional arguments of torch.ops.lightdelta.decode."""
        return (self.qkv, self.a, self.b, self.a_log, self.dt_bias, self.slots, self.cu, self.accepted, self.pool,
                self.gate, self.weight, self.out, self.eps)

    @property
    def num_v_heads(self) -> int:
        return self.pool.shape[1]

    @property
    def tokens(self) -> int:
        return self.qkv.shape[0]


def activation_bytes_per_token(num_k_heads: int, num_v_heads: int) -> int:
    """q + k + v + gate + out (bf16) and a, b (bf16) for one token."""
    qkv = (2 * num_k_heads + num_v_heads) * HEAD_DIM * 2
    gate = out = num_v_heads * HEAD_DIM * 2
    ab = 2 * num_v_heads * 2
    return qkv + gate + out + ab


def decode_algorithmic_bytes(requests: int, width: int, tokens: int, num_k_heads: int, num_v_heads: int,
                             state_itemsize: int = 4) -> int:
    """State read once per request, written once per step, plus activations."""
    slot = num_v_heads * SLOT_HEAD_BYTES * state_itemsize // 4
    return requests * (1 + width) * slot + tokens * activation_bytes_per_token(num_k_heads, num_v_heads)


def make_decode_case(batch: int, width: int, pool_slots: int, *, device, seed: int, num_k_heads: int = 16,
                     num_v_heads: int = 32, accepted: str = "ones", state_scale: float = 0.02,
                     pool: torch.Tensor | None = None) -> DecodeCase:
    """A decode (width 1) or MTP verify (width > 1) case with distinct random slots in 1..pool_slots-1.

    accepted: "ones" (all 1) or "uniform" (U{1..width}).  If `pool` is given it is used as is
    (layer pools shared across cases) and must have `pool_slots` slots.
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    n = batch * width
    hv, h = num_v_heads, num_k_heads
    qkv_width = (2 * h + hv) * HEAD_DIM
    if batch * width > pool_slots - 1:
        raise ValueError("pool too small for distinct slots")
    proj = torch.randn(n, qkv_width + hv * HEAD_DIM, device=device, generator=gen, dtype=torch.float32)
    proj[:, qkv_width:] *= 0.2
    proj = proj.to(torch.bfloat16)
    ba = torch.randn(n, 2 * hv, device=device, generator=gen).to(torch.bfloat16)
    perm = torch.randperm(pool_slots - 1, device=device, generator=gen)[: batch * width] + 1
    slots = perm.to(torch.int32).view(batch, width).contiguous()
    if accepted == "ones":
        acc = torch.ones(batch, device=device, dtype=torch.int32)
    elif accepted == "uniform":
        acc = torch.randint(1, width + 1, (batch,), device=device, generator=gen, dtype=torch.int32)
    else:
        raise ValueError(accepted)
    if pool is None:
        pool = torch.empty(pool_slots, hv, HEAD_DIM, HEAD_DIM, device=device, dtype=torch.float32)
        pool.normal_(0.0, state_scale, generator=gen)
    weight = torch.randn(HEAD_DIM, device=device, generator=gen).to(torch.bfloat16)
    return DecodeCase(
        qkv=proj[:, :qkv_width],
        a=ba[:, hv:],
        b=ba[:, :hv],
        a_log=torch.zeros(hv, device=device, dtype=torch.float32),
        dt_bias=torch.zeros(hv, device=device, dtype=torch.float32),
        slots=slots,
        cu=torch.arange(0, n + 1, width, device=device, dtype=torch.int32),
        accepted=acc,
        pool=pool,
        gate=proj[:, qkv_width:].view(n, hv, HEAD_DIM),
        weight=weight,
        out=torch.empty(n, hv, HEAD_DIM, device=device, dtype=torch.bfloat16),
        num_k_heads=h,
    )


def config2(device, seed: int = 2, pool: torch.Tensor | None = None) -> DecodeCase:
    return make_decode_case(256, 1, 1024, device=device, seed=seed, pool=pool)


def config3(device, seed: int = 3, pool_slots: int = 1 + 256, pool: torch.Tensor | None = None) -> DecodeCase:
    return make_decode_case(64, 4, pool_slots, device=device, seed=seed, accepted="uniform", pool=pool)


@dataclass
class StackedWorkload:
    """BASELINE config 5 on one rank: `layers` decode calls per step over the rank's sequences.

    Every layer has its own seeded activations and weights.  Layer l keeps its states in
    physical pool l % len(pools): when the pools of all 48 layers do not fit in this GPU's
    memory, layers share physical pools (every pool is far larger than L2, so each layer's
    state traffic still comes from HBM).
    """

    layers: list
    pools: list
    sequences: int
    width: int

    def step_bytes(self) -> int:
        c = self.layers[0]
        per_layer = decode_algorithmic_bytes(self.sequences, self.width, c.tokens, c.num_k_heads, c.num_v_heads)
        return per_layer * len(self.layers)


def stacked_workload(device, sequences: int, layers: int = 48, width: int = 4, seed: int = 5,
                     max_pool_bytes: int | None = None, num_k_heads: int = 16,
                     num_v_heads: int = 32, pool_slots: int | None = None) -> StackedWorkload:
    """Config 5: `sequences` local sequences, `width`-token MTP verify, `layers` layers.
    Each physical pool has `pool_slots` slots (default: the null slot plus one per (sequence, step))."""
    slot_bytes = num_v_heads * SLOT_HEAD_BYTES
    if pool_slots is None:
        pool_slots = 1 + sequences * width
    if pool_slots < 1 + sequences * width:
        raise ValueError("pool_slots must hold the null slot and one slot per (sequence, step)")
    pool_bytes = pool_slots * slot_bytes
    physical = layers
    if max_pool_bytes is not None:
        physical = max(1, min(layers, max_pool_bytes // pool_bytes))
    pools = []
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    for _ in range(physical):
        pool = torch.empty(pool_slots, num_v_heads, HEAD_DIM, HEAD_DIM, device=device, dtype=torch.float32)
        pool.normal_(0.0, 0.02, generator=gen)
        pools.append(pool)
    cases = [
        make_decode_case(sequences, width, pool_slots, device=device, seed=seed * 1000 + layer,
                         num_k_heads=num_k_heads, num_v_heads=num_v_heads, accepted="uniform",
                         pool=pools[layer % physical])
        for layer in range(layers)
    ]
    return StackedWorkload(layers=cases, pools=pools, sequences=sequences, width=width)


def config4_indices(device, seed: int = 4, pool_slots: int = 2048, count: int = 512):
    """Gather 512 distinct slots of 1..2047, scatter them to a permutation of another distinct set."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    gather = (torch.randperm(pool_slots - 1, device=device, generator=gen)[:count] + 1).to(torch.int32)
    scatter = (torch.randperm(pool_slots - 1, device=device, generator=gen)[:count] + 1).to(torch.int32)
    return gather, scatter


@dataclass
class SamplingCase:
    """Arguments of torch.ops.lightdelta.greedy_verify over several logits buffers.

    `logits` holds `buffers` independent [rows, vocab] matrices so that cycling through them
    reads more than the 126 MB L2 between two uses of the same buffer.
    """

    logits: list
    cu_num_logits: torch.Tensor
    query_start_loc: torch.Tensor
    input_ids: torch.Tensor
    num_draft_tokens: torch.Tensor
    seq_lens: torch.Tensor
    prefill_len: torch.Tensor
    sampled: torch.Tensor
    num_sampled: torch.Tensor
    num_rejected: torch.Tensor

    def op_args(self, buffer: int) -> tuple:
        return (self.logits[buffer], self.cu_num_logits, self.query_start_loc, self.input_ids,
                self.num_draft_tokens, self.seq_lens, self.prefill_len, self.sampled, self.num_sampled,
                self.num_rejected)

    @property
    def requests(self) -> int:
        return self.num_draft_tokens.numel()

    def bytes_per_launch(self) -> int:
        """Logits rows read (every row is consulted when all requests have steps + 1 rows)."""
        rows, vocab = self.logits[0].shape
        return rows * vocab * self.logits[0].element_size()


def sampling_case(device, seed: int = 6, requests: int = 64, steps: int = 3, vocab: int = 151936,
                  dtype: torch.dtype = torch.float32, buffers: int = 4) -> SamplingCase:
    """Config-3 verification: every request has `steps` drafts and steps + 1 logits rows; a seeded
    prefix of U{0..steps} drafts is planted as the row maximum, the rest of each row is N(0,1)."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    drafts = torch.full((requests,), steps, dtype=torch.int32)
    rows = steps + 1
    cu = torch.arange(0, requests * rows + 1, rows, dtype=torch.int32)
    qsl = cu.clone()  # one accepted token + the drafts per request
    input_ids = torch.randint(0, vocab, (requests * rows,), generator=gen, dtype=torch.int32)
    logits = []
    for b in range(buffers):
        accepted = torch.randint(0, steps + 1, (requests,), generator=gen)
        planted = torch.randint(0, vocab, (requests, rows), generator=gen)
        drafts_of = input_ids.view(requests, rows)[:, 1:]
        for i in range(steps):
            take = accepted > i
            planted[take, i] = drafts_of[take, i].long()
        matrix = torch.empty(requests * rows, vocab, device=device, dtype=torch.float32)
        matrix.normal_(generator=torch.Generator(device=device).manual_seed(seed * 100 + b))
        matrix.view(requests, rows, vocab).scatter_(2, planted.to(device)[:, :, None], 8.0)
        logits.append(matrix.to(dtype))
    return SamplingCase(
        logits=logits,
        cu_num_logits=cu.to(device),
        query_start_loc=qsl.to(device),
        input_ids=input_ids.to(device),
        num_draft_tokens=drafts.to(device),
        seq_lens=torch.full((requests,), 4096, dtype=torch.int32, device=device),
        prefill_len=torch.zeros(requests, dtype=torch.int32, device=device),
        sampled=torch.empty(requests, steps + 1, dtype=torch.int32, device=device),
        num_sampled=torch.empty(requests, dtype=torch.int32, device=device),
        num_rejected=torch.empty(requests, dtype=torch.int32, device=device),
    )


@dataclass
class ConvState:
    """A layer's conv state and conv weights, as vLLM's GDN layer holds them.

    `state` is the [slots, dim, L] view the conv reads ("dim_first": that is the storage;
    "token_first": a transposed view of [slots, L, dim] storage).  L = width - 2 + max tokens.
    """

    state: torch.Tensor
    weight: torch.Tensor
    bias: torch.Tensor | None
    storage: torch.Tensor


def make_conv_state(case: DecodeCase, slots: int, *, seed: int, conv_width: int = 4, layout: str = "dim_first",
                    bias: bool = False) -> ConvState:
    """Seeded bf16 conv state ~ N(0,1), weights ~ 0.5 N(0,1) (and bias ~ 0.1 N(0,1)) for `case`'s
    qkv width; slot 0 is the null block."""
    device = case.qkv.device
    dim = case.qkv.shape[1]
    width = case.slots.shape[1]
    length = conv_width - 2 + width
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    shape = (slots, dim, length) if layout == "dim_first" else (slots, length, dim)
    storage = torch.randn(*shape, device=device, generator=gen).to(torch.bfloat16)
    view = storage if layout == "dim_first" else storage.transpose(1, 2)
    weight = (0.5 * torch.randn(dim, conv_width, device=device, generator=gen)).to(torch.bfloat16)
    b = (0.1 * torch.randn(dim, device=device, generator=gen)).to(torch.bfloat16) if bias else None
    return ConvState(state=view, weight=weight, bias=b, storage=storage)


def conv_decode_args(case: DecodeCase, conv: ConvState) -> tuple:
    """Arguments of torch.ops.lightdelta.conv_decode (case.qkv holds the pre-conv activations)."""
    return (case.qkv, conv.state, conv.weight, conv.bias, case.a, case.b, case.a_log, case.dt_bias, case.slots,
            case.cu, case.accepted, case.pool, case.gate, case.weight, case.out, 1e-6)
