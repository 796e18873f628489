"""GPU parity of torch.ops.lightdelta.conv_update / ld_conv_update (the causal conv1d state update,
vLLM causal_conv1d_update as python/lightdelta/integration/vllm_layer.py:161-172 and :199-207
call it) and conv_decode / ld_conv_decode (that update, then the GDN decode).  Checked against
the CPU oracle (conv restatement pinned to vLLM's kernel, then the decode oracle), against vLLM's
own conv kernel and the unfused pipeline it runs in, and on null conv slots, faults and graph
replay."""

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_out_close_after_conv, assert_state_close_after_conv, bits
from lightdelta_b200 import capi, workloads

pytestmark = pytest.mark.gpu


def host_bf16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def make(device, batch, width, *, heads=(16, 32), layout="dim_first", seed=5, bias=False, pool_slots=None,
         conv_slots=None, accepted="uniform"):
    h, hv = heads
    pool_slots = pool_slots or batch * width + 3
    case = workloads.make_decode_case(batch, width, pool_slots, device=device, seed=seed, num_k_heads=h,
                                      num_v_heads=hv, accepted=accepted if width > 1 else "ones")
    conv = workloads.make_conv_state(case, conv_slots or pool_slots, seed=seed + 1, layout=layout, bias=bias)
    return case, conv


def make_ragged(case, seed):
    """Mixed 1..width tokens per request (vLLM's varlen path: each request's conv state length shrinks
    by the tokens it lacks); the unowned tail rows of qkv stay as they are."""
    batch, width = case.slots.shape
    gen = torch.Generator().manual_seed(seed)
    lengths = torch.randint(1, width + 1, (batch,), generator=gen, dtype=torch.int32)
    lengths[0] = width
    lengths[1] = 1
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lengths, 0)
    case.cu.copy_(cu.to(case.cu.device))
    return case


def oracle_fused(case, conv):
    """Host copies -> oracle conv update -> oracle decode; returns (out bits, pool, conv storage,
    post-conv qkv bits)."""
    qkv = host_bf16(case.qkv)
    state = host_bf16(conv.storage).copy()
    view = state if conv.state.stride(2) == 1 else state.transpose(0, 2, 1)
    slots = case.slots.cpu().numpy()
    cu = case.cu.cpu().numpy()
    post = oracle.conv_update(qkv, view, host_bf16(conv.weight), None if conv.bias is None else host_bf16(conv.bias),
                              slots[:, 0].copy(), case.accepted.cpu().numpy(), cu)
    pool = case.pool.cpu().numpy()
    out = np.zeros(tuple(case.out.shape), np.uint16)
    oracle.decode(post, host_bf16(case.a), host_bf16(case.b), case.a_log.cpu().numpy(), case.dt_bias.cpu().numpy(),
                  slots, cu, case.accepted.cpu().numpy(), pool, host_bf16(case.gate), host_bf16(case.weight), out,
                  num_k_heads=case.num_k_heads)
    return out, pool, state, post


def assert_post_conv_close(got_bits, want_bits):
    """Post-conv activations: bit-exact but for exp rounding (one bf16 ulp, under 1e-3 of values)."""
    diff = np.abs(got_bits.astype(np.int32) - want_bits.astype(np.int32))
    assert diff.max() <= 1, "post-conv values differ by more than one bf16 ulp"
    assert (diff != 0).mean() < 1e-3, f"{(diff != 0).mean():.2e} of post-conv values differ"


@pytest.mark.parametrize("path", ["torch_op", "capi"])
@pytest.mark.parametrize("layout", ["dim_first", "token_first"])
@pytest.mark.parametrize("width", [1, 2, 4])
def test_conv_decode_matches_oracle(device, path, layout, width):
    case, conv = make(device, 24, width, layout=layout, seed=11 + width, bias=width == 2)
    slots = case.slots.clone()
    slots[5, 0] = 0  # null conv slot: the conv is skipped, the decode still runs (if its source is live)
    case.slots.copy_(slots)
    want_out, want_pool, want_state, want_post = oracle_fused(case, conv)
    args = workloads.conv_decode_args(case, conv)
    if path == "torch_op":
        torch.ops.lightdelta.conv_decode(*args)
    else:
        capi.conv_decode(*args)
    torch.cuda.synchronize()
    assert_out_close_after_conv(bits(case.out), want_out, "conv_decode out")
    assert_state_close_after_conv(case.pool.cpu().numpy(), want_pool, "conv_decode pool")
    np.testing.assert_array_equal(host_bf16(conv.storage), want_state)
    assert_post_conv_close(host_bf16(case.qkv), want_post)


@pytest.mark.parametrize("heads", [(16, 16), (16, 32), (16, 48), (8, 32)])
def test_head_geometries(device, heads):
    case, conv = make(device, 6, 4, heads=heads, seed=21)
    want_out, want_pool, want_state, _ = oracle_fused(case, conv)
    torch.ops.lightdelta.conv_decode(*workloads.conv_decode_args(case, conv))
    torch.cuda.synchronize()
    assert_out_close_after_conv(bits(case.out), want_out, f"conv_decode out {heads}")
    assert_state_close_after_conv(case.pool.cpu().numpy(), want_pool, f"conv_decode pool {heads}")
    np.testing.assert_array_equal(host_bf16(conv.storage), want_state)


def test_full_size_config2(device):
    """BASELINE config 2 (256 sequences, HV=32, pool 1024) with a conv state per sequence."""
    case, conv = make(device, 256, 1, pool_slots=1024, seed=2)
    want_out, want_pool, want_state, _ = oracle_fused(case, conv)
    torch.ops.lightdelta.conv_decode(*workloads.conv_decode_args(case, conv))
    torch.cuda.synchronize()
    assert_out_close_after_conv(bits(case.out), want_out, "config 2 out")
    touched = case.slots.flatten().cpu().numpy()
    assert_state_close_after_conv(case.pool[case.slots.flatten().long()].cpu().numpy(), want_pool[touched], "config 2 pool")
    np.testing.assert_array_equal(host_bf16(conv.storage), want_state)


def _vllm_conv():
    try:
        from vllm.model_executor.layers.mamba.ops.causal_conv1d import causal_conv1d_update
    except Exception as exc:  # noqa: BLE001
        pytest.skip(f"vLLM's conv kernel is not importable here: {exc}")
    return causal_conv1d_update


@pytest.mark.parametrize("width", [1, 4])
def test_oracle_conv_matches_vllm_kernel_bf16(device, width):
    """Pins the bf16 arithmetic of the conv oracle to vLLM's compiled kernel on this GPU."""
    causal_conv1d_update = _vllm_conv()
    case, conv = make(device, 64, width, seed=31)
    x = case.qkv.contiguous()
    state_ref = conv.state.clone()
    slots0 = case.slots[:, 0].contiguous()
    if width == 1:
        y = causal_conv1d_update(x.clone(), state_ref, conv.weight, None, "silu", conv_state_indices=slots0,
                                 validate_data=False)
    else:
        y = causal_conv1d_update(x.clone(), state_ref, conv.weight, None, "silu", conv_state_indices=slots0,
                                 num_accepted_tokens=case.accepted, query_start_loc=case.cu, max_query_len=width,
                                 validate_data=False)
    torch.cuda.synchronize()
    host_state = host_bf16(conv.state.contiguous()).copy()
    post = oracle.conv_update(host_bf16(x), host_state, host_bf16(conv.weight), None, slots0.cpu().numpy(),
                              case.accepted.cpu().numpy(), case.cu.cpu().numpy())
    np.testing.assert_array_equal(host_bf16(state_ref.contiguous()), host_state)
    diff = np.abs(host_bf16(y).astype(np.int32) - post.astype(np.int32))
    assert diff.max() <= 1, "post-conv values differ by more than one bf16 ulp"
    assert (diff != 0).mean() < 1e-3, f"{(diff != 0).mean():.2e} of post-conv values differ by one ulp"


@pytest.mark.parametrize("width, ragged", [(1, False), (4, False), (4, True)])
def test_fused_equals_vllm_conv_then_decode(device, width, ragged):
    """The fused op against the pipeline it replaces: vLLM's conv kernel, then lightdelta::decode;
    with `ragged`, requests carry 1..4 tokens."""
    causal_conv1d_update = _vllm_conv()
    case, conv = make(device, 48, width, seed=41)
    if ragged:
        make_ragged(case, 42)
    unfused_pool, unfused_state = case.pool.clone(), conv.state.clone()
    x = case.qkv.clone()
    slots0 = case.slots[:, 0].contiguous()
    if width == 1:
        y = causal_conv1d_update(x, unfused_state, conv.weight, None, "silu", conv_state_indices=slots0,
                                 validate_data=False)
    else:
        y = causal_conv1d_update(x, unfused_state, conv.weight, None, "silu", conv_state_indices=slots0,
                                 num_accepted_tokens=case.accepted, query_start_loc=case.cu, max_query_len=width,
                                 validate_data=False)
    unfused_out = torch.zeros_like(case.out)
    case.out.zero_()  # rows no request owns (ragged case) stay zero in both
    torch.ops.lightdelta.decode(y, case.a, case.b, case.a_log, case.dt_bias, case.slots, case.cu, case.accepted,
                                unfused_pool, case.gate, case.weight, unfused_out, 1e-6)
    torch.ops.lightdelta.conv_decode(*workloads.conv_decode_args(case, conv))
    torch.cuda.synchronize()
    assert torch.equal(conv.state, unfused_state)
    assert_out_close_after_conv(bits(case.out), bits(unfused_out), "fused vs unfused out")
    assert_state_close_after_conv(case.pool.cpu().numpy(), unfused_pool.cpu().numpy(), "fused vs unfused pool")


def test_conv_slot_out_of_range_and_invalid_accepted(device, native):
    """A conv slot out of range: fault bit, the conv skips the request (the decode then sees its
    pre-conv inputs), exactly as if its conv slot were the null block.  accepted outside
    [1, width]: no conv update, zero decode output, decode states untouched."""
    native.fault_flags(clear=True)
    case, conv = make(device, 8, 4, seed=51)
    case.accepted[4] = 0
    base_qkv, base_pool, base_conv = case.qkv.clone(), case.pool.clone(), conv.storage.clone()
    # Reference run: request 2's conv slot is the null block.
    null_slots = case.slots.clone()
    null_slots[2, 0] = 0
    case.slots.copy_(null_slots)
    torch.ops.lightdelta.conv_decode(*workloads.conv_decode_args(case, conv))
    torch.cuda.synchronize()
    want_conv, want_qkv = conv.storage.clone(), case.qkv.clone()
    assert native.fault_flags(clear=True) & native.LD_FAULT_CONV_SLOT_RANGE == 0
    # Run under test: request 2's conv slot is out of range.
    case.qkv.copy_(base_qkv)
    case.pool.copy_(base_pool)
    conv.storage.copy_(base_conv)
    bad_slots = null_slots.clone()
    bad_slots[2, 0] = conv.state.shape[0] + 1
    case.slots.copy_(bad_slots)
    torch.ops.lightdelta.conv_decode(*workloads.conv_decode_args(case, conv))
    torch.cuda.synchronize()
    assert native.fault_flags(clear=True) & native.LD_FAULT_CONV_SLOT_RANGE
    assert torch.equal(conv.storage, want_conv)
    assert torch.equal(case.qkv, want_qkv)
    width = case.slots.shape[1]
    assert not case.out[4 * width:5 * width].any()
    slot = int(case.slots[4, 0])
    assert torch.equal(conv.state[slot], (base_conv if conv.state.stride(2) == 1 else base_conv.transpose(1, 2))[slot])
    for t in range(width):
        s = int(case.slots[4, t])
        assert torch.equal(case.pool[s], base_pool[s])


def test_graph_replay(device):
    case, conv = make(device, 16, 4, seed=61)
    args = workloads.conv_decode_args(case, conv)
    start_qkv, start_pool, start_state = case.qkv.clone(), case.pool.clone(), conv.storage.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        torch.ops.lightdelta.conv_decode(*args)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        torch.ops.lightdelta.conv_decode(*args)
    outs = []
    for _ in range(2):  # replays from the same starting states give identical results
        case.qkv.copy_(start_qkv)
        case.pool.copy_(start_pool)
        conv.storage.copy_(start_state)
        graph.replay()
        torch.cuda.synchronize()
        outs.append((case.out.clone(), case.pool.clone(), conv.storage.clone()))
    assert all(torch.equal(x, y) for x, y in zip(outs[0], outs[1]))
    case.qkv.copy_(start_qkv)
    case.pool.copy_(start_pool)
    conv.storage.copy_(start_state)
    want_out, want_pool, want_state, _ = oracle_fused(case, conv)
    assert_out_close_after_conv(bits(outs[0][0]), want_out, "graph replay out")
    np.testing.assert_array_equal(host_bf16(outs[0][2]), want_state)


@pytest.mark.parametrize("layout", ["dim_first", "token_first"])
@pytest.mark.parametrize("conv_width", [2, 3, 4])
@pytest.mark.parametrize("spec", [False, True])
def test_conv_update_matches_oracle(device, layout, conv_width, spec):
    """conv_update alone: the one-token call (no accepted counts) and the speculative call."""
    width = 4 if spec else 1
    case = workloads.make_decode_case(20, width, 128, device=device, seed=71, accepted="uniform" if spec else "ones")
    conv = workloads.make_conv_state(case, 128, seed=72, conv_width=conv_width, layout=layout, bias=conv_width == 3)
    slots0 = case.slots[:, 0].contiguous()
    slots0[3] = 0
    x = case.qkv.clone()
    host_state = host_bf16(conv.storage).copy()
    view = host_state if layout == "dim_first" else host_state.transpose(0, 2, 1)
    accepted = case.accepted if spec else None
    post = oracle.conv_update(host_bf16(x), view, host_bf16(conv.weight),
                              None if conv.bias is None else host_bf16(conv.bias), slots0.cpu().numpy(),
                              (case.accepted if spec else torch.ones_like(case.accepted)).cpu().numpy(),
                              case.cu.cpu().numpy())
    torch.ops.lightdelta.conv_update(x, conv.state, conv.weight, conv.bias, slots0, accepted, case.cu, width)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bf16(conv.storage), host_state)
    assert_post_conv_close(host_bf16(x), post)


@pytest.mark.parametrize("width, ragged", [(1, False), (4, False), (4, True)])
def test_conv_update_equals_vllm_kernel(device, width, ragged):
    """Our conv kernel against vLLM's on the same GPU: identical state, post-conv values equal
    but for exp rounding; with `ragged`, requests carry 1..4 tokens."""
    causal_conv1d_update = _vllm_conv()
    case, conv = make(device, 64, width, seed=81)
    if ragged:
        make_ragged(case, 82)
    slots0 = case.slots[:, 0].contiguous()
    x_ref, state_ref = case.qkv.contiguous().clone(), conv.state.clone()
    if width == 1:
        y = causal_conv1d_update(x_ref, state_ref, conv.weight, None, "silu", conv_state_indices=slots0,
                                 validate_data=False)
    else:
        y = causal_conv1d_update(x_ref, state_ref, conv.weight, None, "silu", conv_state_indices=slots0,
                                 num_accepted_tokens=case.accepted, query_start_loc=case.cu, max_query_len=width,
                                 validate_data=False)
    x = case.qkv.clone()
    torch.ops.lightdelta.conv_update(x, conv.state, conv.weight, None, slots0, case.accepted if width > 1 else None,
                                     case.cu, width)
    torch.cuda.synchronize()
    assert torch.equal(conv.state, state_ref)
    assert_post_conv_close(host_bf16(x), host_bf16(y))
