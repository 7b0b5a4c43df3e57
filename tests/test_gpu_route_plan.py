"""GPU parity of the routing, the dispatch, the plan and the row dequant, through the C ABI, against the oracle pinned
to the reference (tests/test_oracle.py) and the reference's own golden vectors: ids, counts, permutation, pos and
dequantised values bit-exact; routing weights bit-exact on the reference's exp_nonpos rows (k = 8 softmax) and within
1 ulp of fp32 elsewhere (the GPU's exp() in double against glibc's)."""

import numpy as np
import pytest

from artlite_b200 import CapacityError, Error
from artlite_b200.moe import plan as P
from oracle import moe_np

pytestmark = pytest.mark.gpu


def ulps(a: np.ndarray, b: np.ndarray) -> int:
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return int(np.abs(ia - ib).max()) if a.size else 0


@pytest.mark.parametrize("case", ("E256", "E128"))
def test_route_golden(golden, case):
    lg = golden[f"route_{case}_logits"]
    ids, w = P.route(lg, 8)
    assert np.array_equal(ids, golden[f"route_{case}_cpp_ids"])
    assert np.array_equal(w.view(np.uint32), golden[f"route_{case}_cpp_w"].view(np.uint32))
    assert np.array_equal(ids, golden[f"route_{case}_ref_ids"])
    assert np.abs(w - golden[f"route_{case}_ref_w"]).max() < 2e-7
    E = lg.shape[1]
    assert ids[0, :3].tolist() == [3, 9, E - 56] and ids[1].tolist() == ids[2].tolist() == list(range(8))
    for tag, k, gating in (("_sig6", 6, "sigmoid"), ("_k4", 4, "softmax")):
        ids, w = P.route(lg, k, gating=gating)
        assert np.array_equal(ids, golden[f"route_{case}_cpp{tag}_ids"])
        assert ulps(w, golden[f"route_{case}_cpp{tag}_w"]) <= 1


def test_route_pitched_layout(golden):
    lg = golden["route_E256_logits"]
    rows = np.full((lg.shape[0], 8, 64), np.nan, np.float32)
    rows[:, :, :32] = lg.reshape(lg.shape[0], 8, 32)
    ids, w = P.route(rows.reshape(lg.shape[0], -1), 8, E=256, per_col=32, pitch=64)
    assert np.array_equal(ids, golden["route_pitch_ids"])
    assert np.array_equal(w.view(np.uint32), golden["route_pitch_w"].view(np.uint32))


@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (3, 8, 2), (4096, 128, 8), (777, 64, 6), (100, 1024, 32), (5, 32, 1),
                                   (200, 200, 8)])
def test_route_random_vs_oracle(orc, T, E, k):
    rng = np.random.default_rng(T + E + k)
    lg = (rng.standard_normal((T, E)) * 3).astype(np.float32)
    lg[:, ::7] = np.round(lg[:, ::7])  # (ties)
    if T > 5:
        lg[5, 3] = np.nan
        lg[4, 1] = -np.nan
        lg[2] = -0.0
    for gating in ("softmax", "sigmoid"):
        ids, w = P.route(lg, k, gating=gating)
        rids, rw = orc.route(lg, k, gating=gating)
        assert np.array_equal(ids, rids)
        fin = np.isfinite(rw)
        assert np.array_equal(fin, np.isfinite(w))
        assert ulps(w[fin], rw[fin]) <= 1
        if gating == "softmax" and k == 8 and E % 16 == 0 and E <= 512:  # the exp_nonpos rows: bit-exact
            ok = ~np.isnan(lg).any(1)
            assert np.array_equal(w[ok].view(np.uint32), rw[ok].view(np.uint32))


def test_route_errors():
    with pytest.raises(Error, match="moe_route: k 9 of E 8"):
        P.route(np.zeros((2, 8), np.float32), 9)
    ids, w = P.route(np.zeros((0, 8), np.float32), 2)
    assert ids.shape == (0, 2)


@pytest.mark.parametrize("case", ("T24_E256", "T300_E256", "T200_E128"))
def test_plan_golden(golden, case):
    p = f"plan_{case}_"
    E = int(case.split("_E")[1])
    pl = P.Plan.of(golden[p + "ids"], cap=int(golden[p + "cap"][0]), E=E)
    assert np.array_equal(np.array(pl.counts), golden[p + "counts"])
    assert np.array_equal(pl.pos, golden[p + "pos"])
    for c in range(8):
        n = pl.counts[c]
        assert np.array_equal(pl.experts[c], golden[p + "experts"][c, :n])
        assert np.array_equal(pl.sizes[c], golden[p + "sizes"][c, :n])
        assert np.array_equal(pl.rows[c], golden[p + "rows"][c, :n])


@pytest.mark.parametrize("T", [24, 2048])
def test_plan_reference_properties(T):
    """The reference's own test_plan (tests/moe/test_plan.py:36-57), on the GPU plan."""
    rng = np.random.default_rng(T)
    ids, _ = P.route(rng.standard_normal((T, 256)).astype(np.float32) + np.linspace(0, 3, 256, dtype=np.float32), 8)
    CH, COLS = P.CHUNK, P.COLS
    cap = -(-(256 + -(-T * 8 // CH)) // COLS)
    plan = P.Plan.of(ids, cap=cap, E=256)
    counts = plan.counts
    assert max(counts) - min(counts) <= 1 and sum(counts) == sum(-(-r // CH) for r in np.bincount(ids.ravel()))
    g, j = np.divmod(plan.pos, CH)
    c, k = np.divmod(g, cap)
    assert len(set(plan.pos.ravel().tolist())) == ids.size
    for t in range(T):
        for i in range(8):
            assert plan.experts[c[t, i]][k[t, i]] == ids[t, i] and plan.rows[c[t, i]][k[t, i], j[t, i]] == t
    for col in range(COLS):
        for kk in range(counts[col]):
            r = plan.rows[col][kk]
            n = int(((c == col) & (k == kk)).sum())
            assert (r[n:] == r[0]).all() and (np.diff(r[:n]) > 0).all()


def test_plan_errors(orc):
    ids = np.zeros((4, 2), np.int32)
    ids[3, 1] = 9
    with pytest.raises(Error, match="moe_plan: expert id 9 of 8"):
        P.Plan.of(ids, cap=4, E=8)
    ids = np.arange(64, dtype=np.int32).reshape(32, 2) % 16
    with pytest.raises(CapacityError, match="more than 1 chunks in a column"):
        P.Plan.of(ids, cap=1, E=16, chunk=1)


@pytest.mark.parametrize("T,E,zipf", [(1, 128, 0.0), (16, 128, 0.0), (4096, 128, 1.1), (16384, 128, 0.0),
                                      (3, 8, 0.0), (1000, 1024, 1.1)])
def test_dispatch_vs_oracle(orc, T, E, zipf):
    rng = np.random.default_rng(T)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    if zipf:
        lg += (-zipf * np.log(rng.permutation(E) + 1)).astype(np.float32)
    ids, _ = orc.route(lg, 8)
    off, perm, slot = P.dispatch(ids, E)
    roff, rperm, rslot = orc.dispatch(ids, E)
    assert np.array_equal(off, roff) and np.array_equal(perm, rperm) and np.array_equal(slot, rslot)


@pytest.mark.parametrize("qtype", ("Q4_0", "Q4_1", "Q8_0", "Q4_K", "Q5_K", "Q6_K", "Q3_K", "IQ4_NL", "IQ4_XS"))
def test_dequant_golden(golden, qtype):
    raw, want = golden[f"dq_{qtype}_raw"], golden[f"dq_{qtype}_cpp"]
    got = P.dequant_rows(qtype, raw, want.shape[1])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype", ("Q4_0", "Q8_0", "Q4_K"))
def test_dequant_full_rows(orc, qtype):
    rng = np.random.default_rng(3)
    raw = moe_np.random_blocks(rng, qtype, 64, 2048)
    got = P.dequant_rows(qtype, raw, 2048)
    assert np.array_equal(got.view(np.uint32), orc.dequant_rows(qtype, raw, 2048).view(np.uint32))
