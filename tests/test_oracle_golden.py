"""Pin the CPU oracle (oracle/gh_oracle.py) to fixtures produced by the reference's
own code (tests/golden/make_golden.py). CPU only."""

import numpy as np
import pytest

from oracle import gh_oracle as O


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.mark.parametrize("name,rows,V,seed", [("ce37x257", 37, 257, 11), ("ce16x257", 16, 257, 12), ("ce64x4099", 64, 4099, 13)])
@pytest.mark.parametrize("red", ["sum", "mean"])
@pytest.mark.parametrize("z", [0.0, 1e-4])
def test_ce_oracle_matches_reference(golden, name, rows, V, seed, red, z):
    x, t = O.make_ce_inputs(rows, V, seed, ignore_frac=0.2)
    if f"{name}/logits" in golden.files:
        np.testing.assert_array_equal(golden[f"{name}/logits"], x)
        np.testing.assert_array_equal(golden[f"{name}/target"], t)
    loss = O.cross_entropy_loss(x, t, -100, red, z)
    ref = float(golden[f"{name}/{red}/z{z}/loss"])
    assert abs(loss - ref) <= 1e-5 * max(1.0, abs(ref))
    ce, zs, n, g = O.cross_entropy_with_grad(x, t, z, -100)
    if red == "mean":
        g = g / max(n, 1.0)
    key = f"{name}/{red}/z{z}"
    if f"{key}/grad" in golden.files:
        np.testing.assert_allclose(g, golden[f"{key}/grad"], rtol=1e-4, atol=1e-7)
    else:
        np.testing.assert_allclose(g.reshape(-1)[golden[f"{key}/grad_sel"]], golden[f"{key}/grad_vals"], rtol=1e-4, atol=1e-7)
    assert n == float((t != -100).sum())


@pytest.mark.parametrize("name,shape,seed", [("sls4x16x257", (4, 16, 257), 21), ("sls8x513", (8, 513), 22), ("sls16x151936", (16, 151936), 23)])
def test_sls_oracle_matches_reference(golden, name, shape, seed):
    rows = int(np.prod(shape[:-1]))
    x, idx = O.make_sls_inputs(rows, shape[-1], seed)
    x = x.reshape(shape)
    idx = idx.reshape(shape[:-1])
    out = O.selective_log_softmax(x, idx)
    np.testing.assert_allclose(out, golden[f"{name}/out"], rtol=1e-5, atol=1e-5)
    g = golden[f"{name}/grad_out"]
    grad = O.selective_log_softmax_backward(x, idx, g)
    if f"{name}/grad" in golden.files:
        np.testing.assert_allclose(grad, golden[f"{name}/grad"], rtol=1e-4, atol=1e-6)
    else:
        np.testing.assert_allclose(grad.reshape(-1)[golden[f"{name}/grad_sel"]], golden[f"{name}/grad_vals"], rtol=1e-4, atol=1e-6)


LCE_CASES = [
    ("lce32x128x1000", 32, 128, 1000, 31, 1.0, 0.25, None),
    ("lce37x64x257c11", 37, 64, 257, 32, 1.0, 0.2, 11),
]


@pytest.mark.parametrize("name,N,D,V,seed,wstd,ign,chunk", LCE_CASES)
@pytest.mark.parametrize("red", ["mean", "sum"])
@pytest.mark.parametrize("z", [0.0, 1e-4])
def test_lce_oracle_matches_reference_loop(golden, name, N, D, V, seed, wstd, ign, chunk, red, z):
    H, W, t = O.make_lce_inputs(N, D, V, seed, wstd, ign)
    np.testing.assert_array_equal(golden[f"{name}/H"], H)
    np.testing.assert_array_equal(golden[f"{name}/W"], W)
    loss, dH, dW = O.chunked_linear_cross_entropy(H, W, t, -100, red, z, chunk=chunk)
    key = f"{name}/{red}/z{z}"
    ref = float(golden[f"{key}/loss"])
    assert abs(loss - ref) <= 1e-4 * max(1.0, abs(ref))
    ref_fo = float(golden[f"{key}/loss_fwd_only"])
    lfo = O.chunked_linear_cross_entropy(H, W, t, -100, red, z, chunk=chunk, with_grad=False)
    assert abs(lfo - ref_fo) <= 1e-4 * max(1.0, abs(ref_fo))
    # bf16 results: identical up to rare 1-ulp differences from summation order
    assert rel_l2(dH, golden[f"{key}/grad_H"]) < 5e-3
    assert rel_l2(dW, golden[f"{key}/grad_W"]) < 5e-3
    if f"{key}/test_oracle_loss" in golden.files:
        assert abs(loss - float(golden[f"{key}/test_oracle_loss"])) <= 5e-3 * max(1.0, abs(ref))
        assert rel_l2(dH, golden[f"{key}/test_oracle_grad_H"]) < 5e-2
        assert rel_l2(dW, golden[f"{key}/test_oracle_grad_W"]) < 5e-2


@pytest.mark.parametrize("z", [0.0, 1e-4])
def test_lce_oracle_cfg1_matches_reference(golden, z):
    H, W, t = O.make_lce_inputs(512, 1024, 32000, 0, 0.02, 0.05)
    loss, dH, dW = O.chunked_linear_cross_entropy(H, W, t, -100, "mean", z)
    key = f"cfg1/mean/z{z}"
    ref = float(golden[f"{key}/loss"])
    assert abs(loss - ref) <= 1e-4 * abs(ref)
    assert abs(loss - float(golden[f"{key}/loss_fwd_only"])) <= 1e-4 * abs(ref)
    gh = dH.reshape(-1)[golden[f"{key}/grad_H_sel"]]
    gw = dW.reshape(-1)[golden[f"{key}/grad_W_sel"]]
    assert rel_l2(gh, golden[f"{key}/grad_H_vals"]) < 5e-3
    assert rel_l2(gw, golden[f"{key}/grad_W_vals"]) < 5e-3


def test_chunk_size_matches_reference(golden):
    for B, D, V, elt, ref in golden["chunk_table"]:
        assert O.chunk_size(int(B), int(D), int(V), int(elt)) == int(ref)
