"""The oracle is pinned before it is trusted: the C restatement (oracle/oracle.c) and the NumPy restatement
(oracle/moe_np.py) against the golden vectors that the reference itself wrote (tests/golden/make_golden.py: the
reference's compiled moe_host.cpp / dequant.cpp, its NumPy tests/moe/ref.py, gguf-py), and against the reference's
compiled host code directly when oracle/_ref was built here. CPU only."""

import hashlib

import numpy as np
import pytest

from oracle import lib as olib
from oracle import moe_np

CASES = ("E256", "E128")


@pytest.mark.parametrize("case", CASES)
def test_route_c_oracle_bit_exact(golden, orc, case):
    """ids and fp32 weights equal the reference's compiled moe_route bit for bit (softmax k=8 on its exp_nonpos path,
    sigmoid k=6 and softmax k=4 on std::exp), ties / all-tied / -0 == +0 rows included (test_plan.py:21-26)."""
    lg = golden[f"route_{case}_logits"]
    for tag, k, gating in (("", 8, "softmax"), ("_sig6", 6, "sigmoid"), ("_k4", 4, "softmax")):
        ids, w = orc.route(lg, k, gating=gating)
        assert np.array_equal(ids, golden[f"route_{case}_cpp{tag}_ids"])
        assert np.array_equal(w.view(np.uint32), golden[f"route_{case}_cpp{tag}_w"].view(np.uint32))


@pytest.mark.parametrize("case", CASES)
def test_route_matches_numpy_reference(golden, orc, case):
    """The reference's own agreement (test_plan.py:30-33): ids equal ref.moe_route's, weights within 2e-7; the
    three-way tie and the all-tied row pick the lowest ids."""
    lg = golden[f"route_{case}_logits"]
    ids, w = orc.route(lg, 8)
    assert np.array_equal(ids, golden[f"route_{case}_ref_ids"])
    assert np.abs(w - golden[f"route_{case}_ref_w"]).max() < 2e-7
    E = lg.shape[1]
    assert ids[0, :3].tolist() == [3, 9, E - 56] and ids[1].tolist() == ids[2].tolist() == list(range(8))
    sids, sw = orc.route(lg, 6, gating="sigmoid")
    assert np.array_equal(sids, golden[f"route_{case}_ref_sig6_ids"])
    assert np.abs(sw - golden[f"route_{case}_ref_sig6_w"]).max() < 2e-6


def test_route_pitched_layout(golden, orc):
    """The router GEMM's layout (per column 32 experts at a pitch of 64, NaN padding between columns)."""
    lg = golden["route_E256_logits"]
    rows = np.full((lg.shape[0], 8, 64), np.nan, np.float32)
    rows[:, :, :32] = lg.reshape(lg.shape[0], 8, 32)
    ids, w = orc.route(rows.reshape(lg.shape[0], -1), 8, E=256, per_col=32, pitch=64)
    assert np.array_equal(ids, golden["route_pitch_ids"])
    assert np.array_equal(w, golden["route_pitch_w"])


def test_numpy_route_restatement(golden):
    for case in CASES:
        ids, w = moe_np.moe_route(golden[f"route_{case}_logits"], 8)
        assert np.array_equal(ids, golden[f"route_{case}_ref_ids"])
        assert np.array_equal(w, golden[f"route_{case}_ref_w"])


@pytest.mark.parametrize("case", ("T24_E256", "T300_E256", "T200_E128"))
def test_plan_bit_exact(golden, orc, case):
    p = f"plan_{case}_"
    E = int(case.split("_E")[1])
    ex, counts, sizes, rows, pos = orc.plan(golden[p + "ids"], E=E, cap=int(golden[p + "cap"][0]))
    assert np.array_equal(counts, golden[p + "counts"]) and np.array_equal(pos, golden[p + "pos"])
    for c in range(8):
        n = counts[c]
        assert np.array_equal(ex[c, :n], golden[p + "experts"][c, :n])
        assert np.array_equal(sizes[c, :n], golden[p + "sizes"][c, :n])
        assert np.array_equal(rows[c, :n], golden[p + "rows"][c, :n])


def test_plan_errors(orc):
    """moe_plan's two errors (moe_host.cpp:207, :223): an id outside [0, E) and a column over cap."""
    ids = np.zeros((4, 2), np.int32)
    ids[3, 1] = 9
    with pytest.raises(olib.OracleError):
        orc.plan(ids, E=8, cap=4)
    ids = np.arange(64, dtype=np.int32).reshape(32, 2) % 16
    with pytest.raises(olib.OracleError):
        orc.plan(ids, E=16, cap=1, chunk=1)


def test_dispatch_is_stable_permutation(golden, orc):
    ids = golden["plan_T300_E256_ids"]
    off, perm, slot = orc.dispatch(ids, 256)
    assert off[-1] == ids.size and np.array_equal(np.diff(off), np.bincount(ids.ravel(), minlength=256))
    assert np.array_equal(perm[slot], np.arange(ids.size))
    flat = ids.ravel()
    for e in range(256):
        seg = perm[off[e]:off[e + 1]]
        assert (flat[seg] == e).all() and (np.diff(seg) > 0).all()


@pytest.mark.parametrize("qtype", ("Q4_0", "Q4_1", "Q8_0", "Q4_K", "Q5_K", "Q6_K", "Q3_K", "IQ4_NL", "IQ4_XS"))
def test_dequant_bit_exact(golden, orc, qtype):
    """C and NumPy dequant equal the reference's compiled dequant_rows bit for bit, and gguf-py's values."""
    raw, want = golden[f"dq_{qtype}_raw"], golden[f"dq_{qtype}_cpp"]
    assert np.array_equal(orc.dequant_rows(qtype, raw, want.shape[1]).view(np.uint32), want.view(np.uint32))
    assert np.array_equal(moe_np.dequant(qtype, raw, want.shape[1]).view(np.uint32), want.view(np.uint32))
    np.testing.assert_allclose(want, golden[f"dq_{qtype}_ggufpy"], rtol=1e-6, atol=1e-30)


def test_block_config1(golden, orc):
    """Config 1 (T=16, H=2048, E=128, K=8, F=768, Q4_0, fp32 x, seed 0): the generator reproduces the fixture's
    inputs, and the NumPy moe_ffn with this repository's dequant gives the reference's y (BLAS order aside)."""
    layer, x, _ = moe_np.make_block(0, 16, qtype="Q4_0", x_bf16=False)
    h = hashlib.sha256()
    for arr in (layer.router, x, layer.gate, layer.up, layer.down):
        h.update(np.ascontiguousarray(arr).tobytes())
    assert h.digest() == golden["block_c1_sha256"].tobytes()
    logits = x @ layer.router.T
    ids, w = orc.route(logits, 8)
    assert np.array_equal(ids, golden["block_c1_ids"])
    y = moe_np.moe_ffn(x, ids, w, layer.expert)
    assert moe_np.rel_max(y, golden["block_c1_y"]) < 1e-5


def test_rms_norm_restatement(golden):
    """moe_np.rms_norm (the block's optional input norm) equals the reference's np_ops.rms_norm bit for bit on the
    golden rows (tests/golden/make_golden.py ran the reference's own function)."""
    y = moe_np.rms_norm(golden["norm_x"], golden["norm_w"], 1e-6)
    assert y.dtype == np.float32 and np.array_equal(y.view(np.uint32), golden["norm_y"].view(np.uint32))


def test_against_compiled_reference_when_present(golden, orc):
    """Directly against oracle/_ref (the reference's compiled host code), on fresh random inputs: routing of
    256 x 128 logits with ties and NaNs, the plan of its ids."""
    rl = olib.reference()
    if rl is None:
        pytest.skip("oracle/_ref not built on this host")
    rng = np.random.default_rng(7)
    lg = rng.standard_normal((256, 128)).astype(np.float32)
    lg[5, 7] = np.nan
    lg[6, 3] = -np.nan
    lg[9] = np.round(lg[9])
    for k, gating in ((8, "softmax"), (3, "softmax"), (8, "sigmoid")):
        a, b = orc.route(lg, k, gating=gating), rl.route(lg, k, gating=gating)
        assert np.array_equal(a[0], b[0])
        assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    ids = rl.route(lg, 8)[0]
    cap = -(-(128 + -(-256 * 8 // 192)) // 8)
    for x, y in zip(orc.plan(ids, E=128, cap=cap), rl.plan(ids, E=128, cap=cap)):
        assert np.array_equal(x, y)
