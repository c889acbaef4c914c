"""The causal conv1d oracle against the golden vectors produced by the
reference's own Triton kernels (``tests/golden/make_golden.py``, fixtures
``conv_*.npz``), and a few closed-form properties.  CPU only."""

import glob
import os

import numpy as np
import pytest

from oracle import conv_oracle as C

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "conv_*.npz")))


def _opt(a):
    return None if a.size == 0 else a


def test_fixtures_present():
    names = {os.path.basename(f) for f in FIXTURES}
    for n in ("fla_basic", "fla_init", "fla_varlen", "fn_basic", "fn_short", "fn_null", "fn_apc",
              "upd_basic", "upd_w3", "upd_1nd"):
        assert f"conv_{n}.npz" in names


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[5:-4])
def test_oracle_matches_reference_kernels(path):
    d = np.load(path)
    name = os.path.basename(path)[5:-4]
    act = str(d["activation"]) or None
    if name.startswith("fla"):
        y = C.causal_conv1d(d["x"], d["weight"], _opt(d["bias"]), _opt(d["residual"]),
                            _opt(d["initial_state"]), act, _opt(d["cu_seqlens"]))
        assert np.abs(y - d["y"]).max() < 1e-5
    elif name.startswith("fn"):
        apc = {}
        if "block_idx_last" in d:
            apc = dict(block_idx_first_scheduled_token=d["block_idx_first"],
                       block_idx_last_scheduled_token=d["block_idx_last"],
                       initial_state_idx=d["initial_state_idx"], num_computed_tokens=d["num_computed_tokens"],
                       block_size_to_align=int(d["block_size"]))
        out, cs, proc = C.causal_conv1d_fn(d["x"], d["weight"], _opt(d["bias"]), d["conv_states_in"],
                                           d["query_start_loc"], d["cache_indices"],
                                           d["has_initial_state"], act, **apc)
        qsl = d["query_start_loc"]
        for s in range(len(qsl) - 1):
            if proc[s]:  # skipped sequences are left unwritten by the reference
                np.testing.assert_allclose(out[:, qsl[s]:qsl[s + 1]], d["out"][:, qsl[s]:qsl[s + 1]],
                                           atol=1e-5, rtol=0)
        assert np.array_equal(cs.astype(np.float32), d["conv_states_out"])
    else:
        y, nc = C.causal_conv1d_update(d["x"], d["cache_in"], _opt(d["residual"]), d["weight"],
                                       _opt(d["bias"]), act)
        assert np.abs(y - d["y"]).max() < 1e-5
        assert np.array_equal(nc.astype(np.float32), d["cache_out"])


def test_fn_split_sequence_equals_whole():
    """Running a sequence in two calls, the cache line carrying the state,
    equals one call (the continuous-batching contract)."""
    rng = np.random.default_rng(0)
    dim, W, L = 8, 4, 37
    x = rng.standard_normal((dim, L))
    w = rng.standard_normal((dim, W))
    cs = rng.standard_normal((3, dim, W - 1))
    whole, cs_whole, _ = C.causal_conv1d_fn(x, w, None, cs, [0, L], [2], [True], "silu")
    a, cs_a, _ = C.causal_conv1d_fn(x[:, :10], w, None, cs, [0, 10], [2], [True], "silu")
    b, cs_b, _ = C.causal_conv1d_fn(x[:, 10:], w, None, cs_a, [0, L - 10], [2], [True], "silu")
    np.testing.assert_allclose(np.concatenate([a, b], axis=1), whole, atol=1e-12)
    np.testing.assert_allclose(cs_b, cs_whole, atol=0)


def test_update_steps_equal_fla_forward():
    """Feeding tokens one at a time through the update equals the forward
    with the same starting window."""
    rng = np.random.default_rng(1)
    N, D, W, T = 2, 6, 3, 9
    x = rng.standard_normal((N, T, D))
    w = rng.standard_normal((D, W))
    cache = rng.standard_normal((N, D, W))
    ys = []
    c = cache
    for t in range(T):
        y, c = C.causal_conv1d_update(x[:, t], c, None, w, None, "silu")
        ys.append(y)
    ref = C.causal_conv1d(x, w, None, None, cache, "silu")
    np.testing.assert_allclose(np.stack(ys, 1), ref, atol=1e-12)
