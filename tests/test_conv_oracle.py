"""CPU tests of the conv1d state-update oracle (oracle/conv_oracle.c) against golden fixtures
made by vLLM's own causal_conv1d_update kernel (tests/golden/make_golden_conv.py), the
algorithm the reference calls at python/lightdelta/integration/vllm_layer.py:161-172, :199-207;
and the host-side argument checks of ld_conv_update (nothing is launched)."""

import numpy as np
import pytest

import oracle
from golden import cases

GOLDEN = cases.__file__.rsplit("/", 1)[0]


@pytest.mark.parametrize("spec", cases.CONV_CASES, ids=lambda s: s["name"])
def test_conv_oracle_matches_vllm_kernel(spec):
    case = cases.conv_case(spec)
    golden = np.load(f"{GOLDEN}/{spec['name']}.npz")
    state = case["state"].copy()
    y = oracle.conv_update(case["x"], cases.conv_state_view(spec, state), case["weight"], case["bias"], case["slots"],
                           case["accepted"], case["query_start_loc"])
    # Outputs differ from the kernel's only by the last bit of exp (fp32); states are copies.
    np.testing.assert_allclose(y, golden["y"], rtol=2e-6, atol=1e-6)
    np.testing.assert_array_equal(state[np.unique(case["slots"])], golden["state"])
    skipped = case["slots"] == 0
    qsl = case["query_start_loc"]
    for r in np.flatnonzero(skipped):  # the null conv slot leaves the request's inputs as they were
        np.testing.assert_array_equal(y[qsl[r]:qsl[r + 1]], case["x"][qsl[r]:qsl[r + 1]])


def test_bf16_products_are_rounded():
    """bf16 state and weights: each product is rounded to bf16 before the fp32 accumulation."""
    from golden import detrand

    dim, width = 64, 4
    x = detrand.bf16_bits(detrand.normal(1, (1, dim)))
    state = detrand.bf16_bits(detrand.normal(2, (2, dim, 3)))
    weight = detrand.bf16_bits(detrand.normal(3, (dim, width)))
    y = oracle.conv_update(x, state.copy(), weight, None, [1], [1], [0, 1])
    xs, ss, ws = (detrand.bf16_values(a) for a in (x, state, weight))
    prods = [detrand.bf16_values(detrand.bf16_bits(ss[1, :, j] * ws[:, j])) for j in range(3)]
    prods.append(detrand.bf16_values(detrand.bf16_bits(xs[0] * ws[:, 3])))
    acc = np.zeros(dim, np.float32)
    for p in prods:
        acc = acc + p
    expected = detrand.bf16_bits(acc / (np.float32(1) + np.exp(-acc)))
    assert np.abs(y[0].astype(np.int32) - expected.astype(np.int32)).max() <= 1


@pytest.mark.parametrize("change, message", [
    ({12: 7}, "kernel width"),           # conv_width
    ({18: 5}, "tokens per request"),     # max_tokens
    ({9: 2, 18: 2}, "state length"),     # conv_state_len < width - 2 + max_tokens
    ({3: 0}, "dim >= 1"),                # dim
    ({1: 10}, "invalid strides"),        # x_row_stride < dim
    ({0: None}, "NULL"),                 # x
    ({0: 1 << 20 | 1}, "2-byte aligned"),
    ({6: 100}, "overlap"),               # conv slots closer than one slot's extent
    ({6: 0}, "overlap"),                 # every request on the same slot storage
    ({7: 2}, "overlap"),                 # channels closer than the window length
    ({14: 0}, "invalid strides"),        # slot vector stride 0
])
def test_capi_conv_update_rejects_bad_arguments_before_touching_the_gpu(native, change, message):
    """Host-side checks only: the addresses are never dereferenced (each call fails validation)."""
    fake = 1 << 20
    args = [fake, 64, 4, 64, fake, 8, 192, 3, 1, 3, fake, None, 4, fake, 1, None, fake, 4, 1, None]
    for index, value in change.items():
        args[index] = value
    assert native.lib().ld_conv_update(*args) == native.LD_ERR_INVALID
    assert message in native.last_error()


def test_capi_conv_update_without_requests_is_a_no_op(native):
    args = [None, 64, 0, 64, None, 8, 192, 3, 1, 3, None, None, 4, None, 1, None, None, 0, 1, None]
    assert native.lib().ld_conv_update(*args) == native.LD_OK
