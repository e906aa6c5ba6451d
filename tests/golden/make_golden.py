"""Generate the golden fixtures in this folder from the independent numpy restatement (pyref.py).

Run from the repository root:  python tests/golden/make_golden.py
Writes tests/golden/golden_small.npz. The fixtures pin the C++ oracle (and through it the CUDA
product) to a second, separately written restatement of the reference's encode / plan / scan
arithmetic; the reference ships no golden scan outputs of its own and its Rust toolchain is not
available in this image.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import pyref  # noqa: E402

F = np.float32
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_small.npz")


def queries(doc_seed, n_docs, q_seed, n_q, dims, sigma=0.1):
    noise_seed = pyref.splitmix64(q_seed ^ 0x6E6F697365)
    qs, picks = [], []
    for i in range(n_q):
        p = pyref.splitmix64((q_seed * 0x9E3779B97F4A7C15 + i) & pyref.M64) % n_docs
        x = pyref.synth_row(doc_seed, p, dims)
        q = [F(x[d] + F(F(sigma) * pyref.ih_gauss(noise_seed, i * dims + d))) for d in range(dims)]
        ss = F(0.0)
        for v in q:
            ss = F(ss + F(v * v))
        n = max(np.sqrt(ss), F(1e-12))
        qs.append([F(v / n) for v in q])
        picks.append(p)
    return np.array(qs, np.float32), np.array(picks, np.uint64)


def case(tag, dims, n_docs, n_q, out):
    seed = 42
    docs = np.array([pyref.synth_row(seed, r, dims) for r in range(n_docs)], np.float32)
    out[f"{tag}_docs_sha256"] = np.frombuffer(hashlib.sha256(docs.tobytes()).digest(), np.uint8)
    out[f"{tag}_docs_head"] = docs[:2].copy()
    mean = np.array(pyref.eden_fit(docs, 0, 64), np.float32)
    out[f"{tag}_eden_mean"] = mean
    for codec, cname in ((1, "eden"), (0, "minmax")):
        blocks = []
        for b in range(0, n_docs, 64):
            rows = docs[b:b + 64]
            ts = np.arange(b, b + len(rows), dtype=np.uint32)
            src = np.full(len(rows), 8, np.uint32)
            blocks.append(pyref.encode_block(rows, ts, src, codec, mean, 1))
        blocks = np.concatenate(blocks)
        out[f"{tag}_{cname}_blocks"] = blocks
        qs, picks = queries(seed, n_docs, 7, n_q, dims)
        out[f"{tag}_queries"] = qs
        out[f"{tag}_picks"] = picks
        nb = blocks.size // 4096
        for qi in range(n_q):
            plan = pyref.Plan(qs[qi], codec, mean, 1)
            pre = f"{tag}_{cname}_q{qi}"
            out[pre + "_eden_q_rot"] = np.array(plan.eden_q_rot, np.float32)
            out[pre + "_rabitq_q"] = np.array(plan.rabitq_q, np.float32)
            out[pre + "_w2"] = np.array(plan.w2, np.float32)
            out[pre + "_tfq"] = np.array(plan.tfq, np.float32)
            out[pre + "_tw2"] = np.array(plan.tw2, np.float32)
            out[pre + "_scalars"] = np.array(
                [plan.base, plan.tbase, plan.budget, plan.q_tail_norm, plan.q_mid_norm,
                 plan.q_after_prefix, plan.prefix_sum, plan.eden_mean_ip], np.float32)
            for depth in (0, 1, 2):
                sc = np.zeros(nb * 64, np.float32)
                act = np.zeros(nb * 64, np.uint8)
                for b in range(nb):
                    s = pyref.full_scores_block(blocks[b * 4096:(b + 1) * 4096], plan, depth, 0.2)
                    for v, val in s.items():
                        sc[b * 64 + v] = val
                        act[b * 64 + v] = 1
                out[pre + f"_d{depth}_scores"] = sc
                out[pre + f"_d{depth}_active"] = act


def main():
    out = {}
    # Known-answer values held by the reference's own tests.
    out["kat_lloyd_b4"] = np.array(pyref.B4, np.float32)       # src/eden.rs:27-44
    out["kat_lloyd_b1"] = np.array(pyref.B1, np.float32)       # src/eden.rs:15
    out["kat_offsets"] = np.array([0, 64, 512, 1024, 2048, 2560, 3072, 3584, 4096], np.int64)
    out["kat_crc_check"] = np.array([0xCBF43926], np.uint64)   # CRC-32 check value of b"123456789"
    case("d768", 768, 130, 3, out)
    case("d384", 384, 70, 2, out)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
