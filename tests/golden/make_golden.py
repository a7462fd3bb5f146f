"""Generate the oracle regression fixtures in tests/golden/*.npz.

The reference snapshot has no implementation of this path and no golden
vectors (parity unpinned), so these fixtures pin the CPU oracle itself on
small seeded cases: inputs (storage arrays), summaries and scores in the
canonical fp32 order, the selection, and fp64 outputs. The oracle's stages are
separately checked against the independent numpy twin in tests/test_oracle.py.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT), str(ROOT / "mlx-swift-lm_b200")]

import oracle  # noqa: E402
from sparse_decode.synth import DTYPE_CODE, Workload, make_case  # noqa: E402

CASES = [
    Workload("g_f32_d64", B=1, Hq=8, Hkv=2, D=64, T=600, S=64, K=4, dtype="f32", needles=3),
    Workload("g_bf16_d128", B=1, Hq=4, Hkv=1, D=128, T=515, S=32, K=4, dtype="bf16", needles=3),
    Workload("g_q8_bf16", B=2, Hq=4, Hkv=1, D=128, T=640, S=64, K=3, dtype="bf16", bits=8, needles=2,
             outlier_channels=4, outlier_scale=8.0),
    Workload("g_q4_f16_d64", B=1, Hq=4, Hkv=2, D=64, T=700, S=32, K=6, dtype="f16", bits=4, needles=4),
]


def main() -> None:
    out_dir = Path(__file__).resolve().parent
    for i, w in enumerate(CASES):
        c = make_case(w, seed=1000 + i)
        dt = DTYPE_CODE[w.dtype]
        BH = w.B * w.Hkv
        ks = oracle.to_storage(c["k"].reshape(BH, w.T, w.D), dt)
        vs = oracle.to_storage(c["v"].reshape(BH, w.T, w.D), dt)
        qs = oracle.to_storage(c["q"], dt)
        rec = dict(dtype=dt, B=w.B, Hq=w.Hq, Hkv=w.Hkv, D=w.D, T=w.T, S=w.S, K=w.K, bits=w.bits, q=qs,
                   scale=np.float32(1.0 / np.sqrt(w.D)))
        if w.bits:
            kq = oracle.quantize(ks, dt, w.D, w.bits)
            vq = oracle.quantize(vs, dt, w.D, w.bits)
            Kc = oracle.Cache(dt, w.D, kq[0], w.bits, kq[1], kq[2])
            Vc = oracle.Cache(dt, w.D, vq[0], w.bits, vq[1], vq[2])
            rec.update(k_src=ks, k_wq=kq[0], k_scales=kq[1], k_biases=kq[2], v_wq=vq[0], v_scales=vq[1],
                       v_biases=vq[2])
        else:
            Kc, Vc = oracle.Cache(dt, w.D, ks), oracle.Cache(dt, w.D, vs)
            rec.update(k=ks, v=vs)
        summ = oracle.summaries(Kc, w.T, w.S, dt)
        sc = oracle.scores(qs, dt, summ, dt, w.B, w.Hq, w.Hkv, w.D, w.NB, float(rec["scale"]))
        sel = oracle.select(sc, w.K)
        out = oracle.attend_f64(qs, dt, Kc, Vc, w.B, w.Hq, w.Hkv, w.T, w.S, sel, float(rec["scale"]))
        rec.update(summaries=summ, scores=sc, sel=sel, out=out)
        np.savez_compressed(out_dir / f"{w.name}.npz", **rec)
        print(w.name, "sel", sel.tolist())


if __name__ == "__main__":
    main()
