"""CPU tests of the oracle: pinned against the reference's own results and known answers.

The golden fixtures were produced by running the reference implementation itself
(tests/golden/make_golden.py): post_conv_gdn (python/lightdelta/reference/gdn.py:70-128) and
the Torch-reference packed backend (python/lightdelta/backend.py:30-91) that the reference's
CUDA parity tests use as their expectation.
"""

import numpy as np
import pytest

import oracle
from golden import cases, detrand
from helpers import assert_out_close, assert_state_close, backend_numpy, bf16_values


def _golden(name):
    return np.load(cases.__file__.replace("cases.py", f"{name}.npz"))


@pytest.mark.parametrize("name", [c["name"] for c in cases.POST_CONV_CASES])
def test_oracle_post_conv_matches_reference(name):
    spec = cases.spec_by_name(name)
    x = cases.post_conv_inputs(spec)
    golden = _golden(name)
    output, final, checkpoints = oracle.post_conv_gdn(
        x["q"], x["k"], x["v"], x["a"], x["b"], x["a_log"], x["dt_bias"], x["gate"], x["norm_weight"],
        x["initial_state"], x["lengths"], io_bf16=spec["io_bf16"], save_checkpoints=spec["checkpoints"],
        norm_eps=spec["eps"],
    )
    states = checkpoints if spec["checkpoints"] else final
    assert_state_close(states.reshape(-1)[golden["state_positions"]], golden["state_values"], name)
    if spec["io_bf16"]:
        assert_out_close(detrand.bf16_bits(output), detrand.bf16_bits(golden["output"]), name)
    else:
        np.testing.assert_allclose(output, golden["output"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", [c["name"] for c in cases.BACKEND_CASES])
def test_oracle_decode_matches_reference_backend(name):
    spec = cases.spec_by_name(name)
    x = backend_numpy(spec)
    initial_pool = x["pool"].copy()
    golden = _golden(name)
    oracle.decode(x["qkv"], x["a"], x["b"], x["a_log"], x["dt_bias"], x["slots"], x["cu"], x["accepted"], x["pool"],
                  x["gate"], x["weight"], x["out"], num_k_heads=x["num_k_heads"])
    assert_out_close(x["out"], golden["out_bits"], name)
    assert_state_close(x["pool"].reshape(-1)[golden["pool_positions"]], golden["pool_values"], name)
    np.testing.assert_array_equal(x["pool"][0], initial_pool[0])


def test_scalar_recurrence():
    """Analytic one-dimensional recurrence (reference tests/test_gdn.py:47-55)."""
    one = np.ones((1, 1, 1, 1), np.float32)
    zero = np.zeros((1, 1, 1), np.float32)
    _, final, _ = oracle.post_conv_gdn(one, one, one * 3, zero, zero, np.zeros(1, np.float32),
                                       np.zeros(1, np.float32), one, np.ones(1, np.float32), one * 2,
                                       np.ones(1, np.int64), io_bf16=False)
    key = (1 + 1e-6) ** -0.5
    expected = 1 + 0.5 * (3 - key) * key
    np.testing.assert_allclose(final.reshape(-1), [expected], rtol=1.3e-6, atol=1e-5)


def test_prefix_states_chain_and_masking():
    """T steps at once equal T chained single steps; length 0 leaves the state and zeroes the output
    (reference tests/test_gdn.py:7-44)."""
    spec = cases.spec_by_name("post_conv_small")
    x = cases.post_conv_inputs(spec)
    lengths = x["lengths"]
    names = ("q", "k", "v", "a", "b", "gate")
    common = dict(io_bf16=False)
    original = x["initial_state"].copy()
    full_out, full_final, ckpt = oracle.post_conv_gdn(
        *(x[n] for n in ("q", "k", "v", "a", "b", "a_log", "dt_bias", "gate", "norm_weight", "initial_state")),
        lengths, save_checkpoints=True, **common)
    running = x["initial_state"]
    for t in range(spec["T"]):
        step = {n: x[n][:, t:t + 1] for n in names}
        out, final, _ = oracle.post_conv_gdn(step["q"], step["k"], step["v"], step["a"], step["b"], x["a_log"],
                                             x["dt_bias"], step["gate"], x["norm_weight"], running,
                                             (lengths > t).astype(np.int64), **common)
        np.testing.assert_allclose(out[:, 0], full_out[:, t], rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(final, ckpt[:, t + 1], rtol=1e-6, atol=1e-7)
        running = final
    np.testing.assert_array_equal(x["initial_state"], original)
    np.testing.assert_array_equal(full_final[2], original[2])
    assert np.count_nonzero(full_out[2]) == 0


@pytest.mark.parametrize("index_stride", [1, 4])
def test_oracle_gather_scatter_prefill_semantics(index_stride):
    """Reference tests/test_gdn.py:125-143 restated on the oracle: strided slot vector, zero
    fill for invalid rows, slot 0 untouched."""
    pool = detrand.normal(5, (4, 3, 4, 8), 0.1)
    before = pool.copy()
    storage = np.full((3, index_stride), -1, np.int32)
    slots = storage[:, 0]
    slots[:] = [2, 1, 0]
    valid = np.array([True, False, False])
    packed = np.empty((3, 3, 4, 8), np.float32)
    oracle.gather_state(pool, slots, valid, packed)
    np.testing.assert_array_equal(packed[0], pool[2])
    assert np.count_nonzero(packed[1:]) == 0
    packed += 1
    oracle.scatter_state(packed, slots, pool)
    np.testing.assert_array_equal(pool[0], before[0])
    np.testing.assert_array_equal(pool[1], np.ones_like(pool[1]))
    np.testing.assert_array_equal(pool[2], before[2] + 1)
    np.testing.assert_array_equal(pool[3], before[3])


def test_oracle_copy_slots():
    pool = detrand.normal(6, (6, 2, 4, 4))
    before = pool.copy()
    oracle.copy_slots(pool, np.array([1, 2, 0, 4], np.int32), np.array([3, 2, 5, 0], np.int32))
    np.testing.assert_array_equal(pool[3], before[1])
    for s in (0, 1, 2, 4, 5):
        np.testing.assert_array_equal(pool[s], before[s])


def test_oracle_decode_invalid_requests_write_nothing():
    """Zero output and no state writes for a bad accepted count, a too-long request and an
    out-of-range source; nothing at all for a request without tokens."""
    spec = cases.spec_by_name("backend_hv48_w2")
    x = backend_numpy(spec)
    x["accepted"][:] = [0, 3, 1, 1]        # request 0: accepted 0; request 1: accepted > width
    x["slots"][2, 0] = x["pool"].shape[0]   # request 2: source out of range
    x["cu"][:] = [0, 2, 4, 6, 6]            # request 3: no tokens
    x["out"][:] = 0x3F80                    # 1.0 everywhere, to see what is written
    before = x["pool"].copy()
    oracle.decode(x["qkv"], x["a"], x["b"], x["a_log"], x["dt_bias"], x["slots"], x["cu"], x["accepted"], x["pool"],
                  x["gate"], x["weight"], x["out"], num_k_heads=x["num_k_heads"])
    assert np.count_nonzero(x["out"][:6]) == 0
    assert (bf16_values(x["out"][6:]) == 1.0).all()
    np.testing.assert_array_equal(x["pool"], before)


@pytest.mark.parametrize("name", [c["name"] for c in cases.BACKEND_CASES])
def test_oracle_bf16_pool_is_the_fp32_recurrence_rounded_per_step(name):
    """The bf16-pool mode, pinned to the fp32 mode (itself pinned to the reference): from a pool
    of bf16 values it gives the same outputs as the fp32 pool holding those values widened, and
    stores each step's fp32 state rounded to bf16 (nearest even)."""
    spec = cases.spec_by_name(name)
    x = backend_numpy(spec)
    pool_bits = detrand.bf16_bits(x["pool"])
    x["pool"] = bf16_values(pool_bits)
    y = dict(x, pool=pool_bits.copy(), out=np.zeros_like(x["out"]))
    for args in (x, y):
        oracle.decode(args["qkv"], args["a"], args["b"], args["a_log"], args["dt_bias"], args["slots"], args["cu"],
                      args["accepted"], args["pool"], args["gate"], args["weight"], args["out"],
                      num_k_heads=args["num_k_heads"])
    np.testing.assert_array_equal(y["out"], x["out"])
    np.testing.assert_array_equal(y["pool"], detrand.bf16_bits(x["pool"]))
    assert not np.array_equal(y["pool"], pool_bits)  # some slots were written
