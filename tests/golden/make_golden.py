"""Generates tests/golden/golden.json: small seeded cases run through the CPU oracle.

The reference (Java 25) cannot run in this build environment, so these fixtures pin the
oracle's restatement across changes; the reference's own known-answer values live in
tests/test_oracle_golden.py.  Regenerate with:  python -m tests.golden.make_golden
"""
import json
import os

import numpy as np


def _bits(a):
    return [int(x) for x in np.asarray(a, np.float32).view(np.uint32).reshape(-1)]


def compute(O):
    out = {}
    db = O.gen_mixture(2000, 96, 8, 0.3, 0xC0FFEE03, 0xC0FFEE01, True)
    q = O.gen_mixture(6, 96, 8, 0.3, 0xC0FFEE03, 0xC0FFEE02, True)
    out["mixture_checksum"] = _bits(db.sum(axis=1))[:16]
    for metric in range(4):
        ids, sc, cnt = O.flat_search(db, q, metric, 10)
        out[f"flat_{metric}"] = {"ids": ids.tolist(), "scores": _bits(sc), "counts": cnt.tolist()}
    lo, hi = O.sq8_train(db)
    codes, corr = O.sq8_encode_all(lo, hi, db)
    out["sq8_quantiles"] = _bits([lo, hi])
    out["sq8_corr_head"] = _bits(corr[:16])
    for metric in range(4):
        ids, sc, cnt = O.sq8_search(codes, corr, lo, hi, q, metric, 10)
        out[f"sq8_{metric}"] = {"ids": ids.tolist(), "scores": _bits(sc)}
    words = O.bq_encode_all(db)
    for metric in range(4):
        ids, sc, cnt = O.bq_search(words, 96, q, metric, 10)
        out[f"bq_{metric}"] = {"ids": ids.tolist(), "scores": _bits(sc)}
    f16 = O.fp16_encode_all(db)
    ids, sc, cnt = O.fp16_search(f16, q, O.DOT_PRODUCT, 10)
    out["fp16_1"] = {"ids": ids.tolist(), "scores": _bits(sc)}
    cb = O.pq_train(db, 12, 16)
    out["pq_codebook_head"] = _bits(cb[:32])
    cent = O.kmeans_train(db, 16, 10, 42)
    assign = O.kmeans_assign(db, cent)
    off, ords = O.build_ivf_lists(assign, 16)
    resid = db - cent[assign]
    cb2 = O.pq_train(resid, 12, 16)
    pq = O.pq_encode_all(resid, 12, 16, cb2)
    ids, sc, cnt = O.ivfpq_search(cent, off, ords, 12, 16, cb2, pq, q, O.EUCLIDEAN, 10, 4)
    out["ivfpq_0"] = {"ids": ids.tolist(), "scores": _bits(sc)}
    # routing, the IVF-flat batched scan, the cluster radii, SQ4 and BBQ
    for metric in range(4):
        lids, dists = O.route(cent, q, metric, 5)
        out[f"route_{metric}"] = {"ids": lids.tolist(), "dists": _bits(dists)}
        ids, sc, cnt = O.ivfflat_search(cent, off, ords, db, q, metric, 10, 4)
        out[f"ivfflat_{metric}"] = {"ids": ids.tolist(), "scores": _bits(sc), "counts": cnt.tolist()}
    out["ivf_radii"] = _bits(O.ivf_radii(cent, off, ords, db))
    packed, corr4 = O.sq4_encode_all(lo, hi, db)
    out["sq4_corr_head"] = _bits(corr4[:16])
    for metric in range(2):
        ids, sc, cnt = O.sq4_search(packed, corr4, 96, lo, hi, q, metric, 10)
        out[f"sq4_{metric}"] = {"ids": ids.tolist(), "scores": _bits(sc)}
    c0 = db.mean(0).astype(np.float32)
    bw, bc = O.bbq_encode_all(db, c0)
    out["bbq_corr_head"] = _bits(bc[:8])
    for metric in range(4):
        ids, sc, cnt = O.bbq_search(bw, bc, c0, 96, q, metric, 10)
        out[f"bbq_{metric}"] = {"ids": ids.tolist(), "scores": _bits(sc)}
    return out


if __name__ == "__main__":
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    from oracle import oracle as O

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    with open(path, "w") as f:
        json.dump(compute(O), f, separators=(",", ":"))
    print("wrote", path, os.path.getsize(path), "bytes")
