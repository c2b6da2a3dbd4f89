"""The CPU oracle against the reference's own recorded outputs.

tests/golden/reference_examples.json holds, for each pinned playground example
(runtime/playground/example-results.json), the value the reference recorded in
its browser run and the value the unmodified reference package produced on the
oracle through the shim (tests/golden/make_golden.py).  The RNG example is
bit-exact (integer xorshift + one rounding); transcendental paths carry the
ulp differences between the browser's WGSL math and the host libm.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "reference_examples.json")))

# relative tolerance per example: rand is bit-exact; randn goes through
# log/sqrt/cos; autograd_conv2d sums randn values.
# nn_linear_relu draws its weights and input with randn (log / sqrt / cos) and
# sums 8 products; unary_sqrt_exp_log's log(2.718281828) is 1 ulp from 1.0.
RTOL = {"rand_tensor": 0.0, "randn_tensor": 2e-6, "autograd_conv2d": 2e-6, "nn_linear_relu": 2e-6,
        "unary_sqrt_exp_log": 2e-7}
ATOL = {"nn_linear_relu": 1e-7, "unary_sqrt_exp_log": 1e-7}
UNPINNED = json.load(open(os.path.join(HERE, "golden", "recorded_unpinned.json")))


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_oracle_matches_reference_recording(name):
    g = GOLDEN[name]
    rtol, atol = RTOL.get(name, 0.0), ATOL.get(name, 0.0)
    for key in g["keys"]:
        rec, got = g["recorded"][key], g["oracle"][key]
        if g.get("kat"):  # the browser suite's known answer, compared at its own precision
            atol = g["tol"][key]
        if isinstance(rec, (list, float, int)) and not isinstance(rec, bool):
            a = np.asarray(rec, dtype=np.float64)
            b = np.asarray(got, dtype=np.float64)
            assert a.shape == b.shape, (name, key)
            np.testing.assert_allclose(b, a, rtol=rtol, atol=atol, err_msg=f"{name}.{key}")
        else:
            assert rec == got, (name, key)


def test_seeded_examples_record_their_seed():
    """nn_linear_relu (nn.Linear's Kaiming-uniform init and a randn input)
    reproduces its recording from one starting seed of the playground session."""
    assert GOLDEN["nn_linear_relu"]["seed"] is not None and GOLDEN["nn_linear_relu"]["seed"] >= 42


def test_unpinned_recordings_disagree_with_the_shader_arithmetic():
    """The recordings kept out of the pins: where the recording contradicts the
    shader's own arithmetic on the script's input, the oracle gives that
    arithmetic (numpy recomputes it here)."""
    am = UNPINNED["argmax_argmin"]
    x = np.asarray(am["oracle"]["input"])
    assert am["oracle"]["argmax"] == np.argmax(x, axis=1).tolist()
    assert am["oracle"]["argmin"] == np.argmin(x, axis=1).tolist()
    assert am["recorded"]["argmax"] != am["oracle"]["argmax"]
    rd = UNPINNED["reduce_dim_keepdim"]
    xs = np.array([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
    assert rd["oracle"]["sum(0, keepdim)"] == xs.sum(axis=0, keepdims=True).tolist()
    assert rd["oracle"]["mean(1, keepdim)"] == xs.mean(axis=1, keepdims=True).tolist()
    assert all(v.get("why") for v in UNPINNED.values())


def test_oracle_rand_reproduces_recording_directly():
    """rand at the initial seed 42 (creationOps.ts:17) restated in C is bit-exact."""
    import oracle_runtime as O
    vals = O.random(6, 42, 0)
    rec = np.asarray(GOLDEN["rand_tensor"]["recorded"]["values"], np.float32).reshape(-1)
    assert np.array_equal(vals, rec)


def test_tiny_cnn_trace_replays_on_oracle_in_ten_steps():
    """bench.py --workload tiny splits the recorded Tiny-CNN stream into its 10
    training steps; replayed on the oracle it reproduces every recorded
    readback exactly (the stream was recorded on the oracle)."""
    import importlib.util
    import sys
    root = os.path.dirname(HERE)
    sys.path.insert(0, os.path.join(root, "oracle"))
    from oracle_runtime import OracleRuntime
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    calls = json.load(open(bench.TINY_TRACE))["calls"]
    times, dev = bench.replay_trace(OracleRuntime(), calls)
    assert len(times) == 10 and all(t > 0 for t in times)
    assert dev == 0.0
