"""A second, independent restatement (numpy float32, one Java operation at a time) of the oracle
paths that have no golden vectors from the reference: SQ4 encoding and scoring
(ScalarQuantizer.java:59-69,243-351, ScalarQuantizedVectors.java:110-140), BBQ encoding and
scoring (BinaryQuantizer.java:207-270, BinaryQuantizedVectors.java:110-275) and the IVF-flat
scan (IvfIndex.java:170-277).  The C++ oracle must agree with it to the bit on small cases."""
import numpy as np
import pytest

f32 = np.float32


def java_round(x):
    """Math.round(float): floor(x + 0.5) for finite x (ties toward +infinity)."""
    return int(np.floor(np.float64(x) + 0.5))


def sq_consts(lo, hi, max_value):
    rng = f32(f32(hi) - f32(lo))
    scale = f32(0) if rng == 0 else f32(f32(max_value) / rng)
    alpha = f32(0) if rng == 0 else f32(rng / f32(max_value))
    return scale, alpha, f32(alpha * alpha)


def sq_encode(v, lo, hi, max_value):
    scale, alpha, _ = sq_consts(lo, hi, max_value)
    lo, hi = f32(lo), f32(hi)
    codes, corr = [], f32(0)
    for x in v.astype(f32):
        dxc = f32(max(lo, min(hi, x)) - lo)
        q = max(0, min(max_value, java_round(f32(scale * dxc))))
        codes.append(q)
        dx = f32(x - lo)
        dxq = f32(f32(q) * alpha)
        t1 = f32(lo * f32(x - f32(lo / f32(2))))
        t2 = f32(f32(dx - dxq) * dxq)
        corr = f32(corr + f32(t1 + t2))
    return np.array(codes, np.int64), corr


def sq_score(metric, qc, qcorr, vc, vcorr, lo, hi, max_value):
    _, _, cm = sq_consts(lo, hi, max_value)
    if metric == 0:
        sq = int(((qc - vc) ** 2).sum())
        return f32(f32(1) / f32(f32(1) + f32(f32(sq) * cm)))
    raw = int((qc * vc).sum())
    adj = f32(f32(f32(f32(raw) * cm) + qcorr) + vcorr)
    if metric == 3:
        return None  # MIP goes through scaleMaxInnerProductScore, pinned elsewhere
    return max(f32(f32(f32(1) + adj) / f32(2)), f32(0))


def test_sq4_encode_and_scores_match_a_second_restatement(oracle):
    rng = np.random.default_rng(11)
    db = rng.standard_normal((40, 23)).astype(np.float32)
    q = rng.standard_normal((3, 23)).astype(np.float32)
    lo, hi = oracle.sq8_train(db)
    packed, corr = oracle.sq4_encode_all(lo, hi, db)
    codes = oracle.sq4_unpack(packed, 23).astype(np.int64)
    for i in range(len(db)):
        c, k = sq_encode(db[i], lo, hi, 15)
        assert np.array_equal(c, codes[i]) and k == corr[i], f"row {i}"
    for metric in (0, 1):
        ids, sc, cnt = oracle.sq4_search(packed, corr, 23, lo, hi, q, metric, 40)
        for j in range(len(q)):
            qc, qk = sq_encode(q[j], lo, hi, 15)
            for r in range(cnt[j]):
                o = ids[j, r]
                assert sc[j, r] == sq_score(metric, qc, qk, codes[o], corr[o], lo, hi, 15), (metric, j, r)


def bbq_encode(v, c):
    cc = (v.astype(f32) - c.astype(f32)).astype(f32)
    dist = f32(0)
    for x in cc:
        dist = f32(dist + f32(x * x))
    bits = (cc >= 0).astype(np.int64)
    return bits, (dist, f32(cc.min()), f32(f32(cc.max()) - f32(cc.min())))


def bbq_score(metric, qv, cent, bits, corr):
    c = (qv.astype(f32) - cent.astype(f32)).astype(f32)
    nsq = f32(0)
    for x in c:
        nsq = f32(nsq + f32(x * x))
    mn, mx = f32(c.min()), f32(c.max())
    width = f32(mx - mn)
    scale = f32(f32(15) / width) if width > 0 else f32(0)
    q4 = np.array([max(0, min(15, java_round(f32(f32(x - mn) * scale)))) for x in c], np.int64)
    qsum = int(q4.sum())
    raw = int((q4 * bits).sum())
    pop = int(bits.sum())
    dist, vl, w = corr
    dim = len(c)
    approx = f32(f32(mn * f32(f32(vl * f32(dim)) + f32(w * f32(pop))))
                 + f32(f32(width / f32(15)) * f32(f32(vl * f32(qsum)) + f32(w * f32(raw)))))
    if metric == 1:
        return max(f32(f32(f32(1) + approx) / f32(2)), f32(0))
    if metric == 0:
        adj = f32(f32(nsq + dist) - f32(f32(2) * approx))
        return f32(f32(1) / f32(f32(1) + max(adj, f32(0))))
    norm = f32(np.sqrt(np.float64(nsq)))
    vn = f32(np.sqrt(np.float64(dist)))
    if norm == 0 or vn == 0:
        return f32(0)
    cosv = f32(approx / f32(norm * vn))
    return max(f32(f32(f32(1) + cosv) / f32(2)), f32(0))


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_bbq_encode_and_scores_match_a_second_restatement(oracle, metric):
    rng = np.random.default_rng(12)
    db = rng.standard_normal((30, 70)).astype(np.float32)
    q = rng.standard_normal((3, 70)).astype(np.float32)
    cent = db.mean(0).astype(np.float32)
    words, corr = oracle.bbq_encode_all(db, cent)
    for i in range(len(db)):
        bits, cr = bbq_encode(db[i], cent)
        packed = np.zeros(2, np.uint64)
        for d in np.nonzero(bits)[0]:
            packed[d >> 6] |= np.uint64(1) << np.uint64(d & 63)
        assert np.array_equal(packed, words[i]) and tuple(corr[i]) == cr, f"row {i}"
    ids, sc, cnt = oracle.bbq_search(words, corr, cent, 70, q, metric, 30)
    for j in range(len(q)):
        for r in range(cnt[j]):
            o = ids[j, r]
            bits, cr = bbq_encode(db[o], cent)
            assert sc[j, r] == bbq_score(metric, q[j], cent, bits, cr), (metric, j, r)


def mat_vec_l2(q, rows):
    """matVecSquaredL2 over a batch: rows in groups of four on 8 lane accumulators (FMA), the
    batch's last count % 4 rows through squareDistance (taken from the oracle's scalar form)."""
    out = []
    dim = len(q)
    limit = dim & ~7
    for r in range(len(rows) & ~3):
        acc = [f32(0)] * 8
        for i in range(0, limit, 8):
            for j in range(8):
                d = f32(q[i + j] - rows[r][i + j])
                # fused multiply-add through float64: d * d is exact there; the sum rounds twice
                # (float64 then float32), which could differ from one rounding only at
                # exponent gaps these small sums do not reach
                acc[j] = f32(np.float64(d) * np.float64(d) + np.float64(acc[j]))
        lanes = acc
        even = f32(f32(lanes[4] + lanes[0]) + f32(lanes[6] + lanes[2]))
        odd = f32(f32(lanes[5] + lanes[1]) + f32(lanes[7] + lanes[3]))
        s = f32(even + odd)
        for i in range(limit, dim):
            e = f32(q[i] - rows[r][i])
            s = f32(np.float64(e) * np.float64(e) + np.float64(s))
        out.append(s)
    return out


def test_ivfflat_batched_scores_match_a_second_restatement(oracle):
    # one list, every row probed: the oracle's IVF-flat EUCLIDEAN scores of the batch-arithmetic
    # rows equal -matVecSquaredL2 restated here (dims not a multiple of 8: the folded tail)
    rng = np.random.default_rng(13)
    db = rng.standard_normal((70, 21)).astype(np.float32)
    q = rng.standard_normal((1, 21)).astype(np.float32)
    cent = db.mean(0, keepdims=True).astype(np.float32)
    off = np.array([0, 70], np.int64)
    ords = np.arange(70, dtype=np.int32)
    ids, sc, cnt = oracle.ivfflat_search(cent, off, ords, db, q, 0, 70, 1)
    batch = mat_vec_l2(q[0], db[:64])  # the first batch: 64 rows, all in groups of four
    got = {int(i): s for i, s in zip(ids[0, : cnt[0]], sc[0, : cnt[0]])}
    for r in range(64):
        assert got[r] == -batch[r], r
