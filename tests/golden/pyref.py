"""Independent pure-numpy restatement of the reference PaxBlock64 path, for SMALL cases only.

This is a second, separately written restatement of the reference crate `mrl_index` v0.3.5
(paths relative to its project root) used to generate the golden fixtures in this folder and to
cross-check the C++ oracle. It shares no code with the oracle: binary16 conversion comes from
numpy's float16 (IEEE round-to-nearest-even, the `half` crate's semantics), CRC-32 from zlib
(the `crc32fast` algorithm), and every f32 operation is an explicit numpy float32 scalar op so
it rounds where the Rust code rounds. Sequential sums are explicit loops (the reference never
reassociates).
"""
from __future__ import annotations

import math
import struct
import zlib

import numpy as np

F = np.float32
M64 = (1 << 64) - 1

B1 = [F(-0.79788456), F(0.79788456)]  # src/eden.rs:15
B4 = [F(v) for v in (-2.73258958, -2.06901724, -1.61804640, -1.25623121, -0.94234046,
                     -0.65675912, -0.38804830, -0.12839503, 0.12839503, 0.38804830,
                     0.65675912, 0.94234046, 1.25623121, 1.61804640, 2.06901724,
                     2.73258958)]  # src/eden.rs:27-44
PI_F = F(math.pi)


def sign_hash(a: int, i: int) -> F:
    """tail_rademacher (src/rotate.rs:53-67) / rademacher_diag (src/eden.rs:75-88)."""
    x = (((a * 0x9E3779B97F4A7C15) & M64) + i) & M64
    x = (x * 0xBF58476D1CE4E5B9) & M64
    x ^= x >> 30
    x = (x * 0x94D049BB133111EB) & M64
    x ^= x >> 27
    return F(1.0) if x & 1 == 0 else F(-1.0)


def fwht(a):
    """fwht_inplace, src/rotate.rs:13-33."""
    a = [F(v) for v in a]
    n = len(a)
    h = 1
    while h < n:
        for i in range(0, n, 2 * h):
            for j in range(i, i + h):
                x, y = a[j], a[j + h]
                a[j] = F(x + y)
                a[j + h] = F(x - y)
        h *= 2
    scale = F(F(1.0) / np.sqrt(F(n)))
    return [F(v * scale) for v in a]


def rabitq_bit_scale():
    return F(np.sqrt(F(F(2.0) / PI_F)) / np.sqrt(F(128.0)))


def tail_fold_bit_scale():
    return F(np.sqrt(F(F(2.0) / PI_F)) / np.sqrt(F(64.0)))


def rotate_tail_fold(vec):
    """fold_tail + FWHT64, src/rotate.rs:73-100."""
    u = [F(0.0)] * 64
    if len(vec) > 192:
        nb = min((len(vec) - 192) // 64, 9)
        for b in range(nb):
            base = 192 + 64 * b
            for d in range(64):
                u[d] = F(u[d] + F(sign_hash(b, d) * F(vec[base + d])))
    return fwht(u)


def round_half_away(x: F) -> float:
    v = float(x)
    r = math.floor(abs(v) + 0.5)
    return math.copysign(r, v)


def nearest_centroid(cb, z):
    """src/eden.rs:57-71."""
    lo = 0
    hi = len(cb)
    while lo < hi:
        mid = (lo + hi) // 2
        if cb[mid] < z:
            lo = mid + 1
        else:
            hi = mid
    if lo < len(cb) and cb[lo] == z:
        return lo
    if lo == 0:
        return 0
    if lo >= len(cb):
        return len(cb) - 1
    return lo - 1 if abs(F(z - cb[lo - 1])) <= abs(F(cb[lo] - z)) else lo


def eden_encode_slice(mean, seed, cb, x):
    """encode_slice, src/eden.rs:225-269."""
    d = len(mean)
    sqrt_d = np.sqrt(F(d))
    inv_sqrt_d = F(F(1.0) / sqrt_d)
    c = []
    ns = F(0.0)
    for i in range(d):
        v = F(F(x[i]) - mean[i])
        c.append(v)
        ns = F(ns + F(v * v))
    cn = max(np.sqrt(ns), F(1e-12))
    inv = F(F(1.0) / cn)
    c = [F(v * inv) for v in c]
    c = [F(c[i] * sign_hash(seed, i)) for i in range(d)]
    c = fwht(c)
    levels = []
    ip = F(0.0)
    for i in range(d):
        lv = nearest_centroid(cb, F(c[i] * sqrt_d))
        levels.append(lv)
        ip = F(ip + F(c[i] * F(cb[lv] * inv_sqrt_d)))
    ss = F(F(1.0) / ip) if abs(ip) > F(1e-12) else F(0.0)
    return levels, cn, ss


def f16_bits(x) -> int:
    return int(np.array([x], dtype=np.float32).astype(np.float16).view(np.uint16)[0])


def f16_val(bits: int) -> F:
    return F(np.array([bits], np.uint16).view(np.float16)[0])


def eden_fit(rows, start, width):
    """EdenFit::fit_band, src/eden.rs:130-161."""
    mean = [F(0.0)] * width
    for r in rows:
        for d in range(width):
            mean[d] = F(mean[d] + F(r[start + d]))
    inv = F(F(1.0) / F(len(rows)))
    return [F(m * inv) for m in mean]


def encode_block(vecs, ts, src, prefix_codec, eden_mean=None, eden_seed=1):
    """encode_block_with_fits (src/quantize.rs:36-96), Rabitq mid band only."""
    blk = bytearray(4096)
    planes = {o: [0] * n for o, n in ((512, 64), (1024, 128), (2048, 64), (2560, 64), (3072, 64), (3584, 64))}
    n = len(vecs)
    for i, v in enumerate(vecs):
        v = [F(x) for x in v]
        dims = len(v)
        if prefix_codec == 1:
            levels, cn, ss = eden_encode_slice(eden_mean, eden_seed, B4, v[:64])
            scale, offset = F(cn * ss), F(0.0)
        else:  # quantize_vector, src/quantize.rs:220-246
            mn, mx = F(np.inf), F(-np.inf)
            for x in v[:64]:
                mn, mx = min(mn, x), max(mx, x)
            rng = max(F(mx - mn), F(1e-8))
            scale = F(rng / F(15.0))
            offset = mn
            levels = [int(min(max(round_half_away(F(F(x - offset) / scale)), 0.0), 15.0)) for x in v[:64]]
        rot = fwht(v[64:192])
        rab = [1 if r >= 0 else 0 for r in rot]
        fold = [1 if r >= 0 else 0 for r in rotate_tail_fold(v)]
        mid_sq = F(0.0)
        for x in v[64:192]:
            mid_sq = F(mid_sq + F(x * x))
        high_sq = F(0.0)
        for x in v[192:]:
            high_sq = F(high_sq + F(x * x))
        rest = np.sqrt(F(mid_sq + high_sq))
        high = np.sqrt(high_sq)
        if rest <= F(1e-12):
            flags = 0
        else:
            r = min(max(F(high / rest), F(0.0)), F(1.0))
            flags = int(min(max(round_half_away(F(r * F(255.0))), 0.0), 255.0))
        struct.pack_into("<HHHB", blk, 64 + 7 * i, f16_bits(scale), f16_bits(offset), f16_bits(rest), flags)
        for d in range(64):
            q = levels[d]
            if q & 8: planes[512][d] |= 1 << i
            if q & 4: planes[2048][d] |= 1 << i
            if q & 2: planes[2560][d] |= 1 << i
            if q & 1: planes[3584][d] |= 1 << i
        for d in range(128):
            if rab[d]: planes[1024][d] |= 1 << i
        for d in range(64):
            if fold[d]: planes[3072][d] |= 1 << i
    for off, words in planes.items():
        struct.pack_into(f"<{len(words)}Q", blk, off, *words)
    tomb = 0
    for i in range(n, 64):
        tomb |= 1 << i
    struct.pack_into("<IIIHHQI", blk, 0, min(ts), max(ts), int(np.bitwise_or.reduce(src)), 0, 0, tomb, 0)
    crc = zlib.crc32(bytes(blk)) & 0xFFFFFFFF
    struct.pack_into("<I", blk, 24, crc)
    return np.frombuffer(bytes(blk), np.uint8).copy()


class Plan:
    """QueryPlan::from_query_codec (src/scan.rs:105-266), Rabitq mid band."""

    def __init__(self, q, prefix_codec, eden_mean=None, eden_seed=1):
        q = [F(x) for x in q]
        dims = len(q)
        self.prefix_codec = prefix_codec
        self.prefix = q[:64]
        s = F(0.0)
        for x in self.prefix:
            s = F(s + x)
        self.prefix_sum = s
        self.bw3 = [F(x * F(8.0)) for x in self.prefix]
        self.eden_inv_sqrt_d = F(F(1.0) / np.sqrt(F(64.0)))
        self.eden_q_rot = [F(0.0)] * 64
        self.eden_mean_ip = F(0.0)
        if prefix_codec == 1:
            rot = [F(q[i] * sign_hash(eden_seed, i)) for i in range(64)]
            self.eden_q_rot = fwht(rot)
            ip = F(0.0)
            for d in range(64):
                ip = F(ip + F(q[d] * eden_mean[d]))
            self.eden_mean_ip = ip
        self.rabitq_q = fwht(q[64:192])
        sc = rabitq_bit_scale()
        base = F(0.0)
        self.w2 = []
        for d in range(128):
            pos = F(self.rabitq_q[d] * sc)
            base = F(base - pos)
            self.w2.append(F(F(2.0) * pos))
        self.base = base
        tsq = F(0.0)
        for x in q[192:]:
            tsq = F(tsq + F(x * x))
        self.q_tail_norm = np.sqrt(tsq)
        msq = F(0.0)
        for x in q[64:192]:
            msq = F(msq + F(x * x))
        self.q_mid_norm = np.sqrt(msq)
        self.q_after_prefix = np.sqrt(F(msq + tsq))
        self.has_tail_fold = dims > 192
        self.tfq = rotate_tail_fold(q) if self.has_tail_fold else [F(0.0)] * 64
        ts = tail_fold_bit_scale()
        tb, bud = F(0.0), F(0.0)
        self.tw2 = [F(0.0)] * 64
        if self.has_tail_fold:
            for d in range(64):
                pos = F(self.tfq[d] * ts)
                tb = F(tb - pos)
                self.tw2[d] = F(F(2.0) * pos)
                bud = F(bud + abs(pos))
        self.tbase = tb
        self.budget = bud


def decode_meta(blk, v):
    sc, off, tn, fl = struct.unpack_from("<HHHB", bytes(blk[64 + 7 * v: 71 + 7 * v]))
    scale, offset, tail = f16_val(sc), f16_val(off), f16_val(tn)
    rho = F(F(fl) / F(255.0))
    t = max(tail, F(0.0))
    r = min(max(rho, F(0.0)), F(1.0))
    mid = F(np.sqrt(max(F(F(1.0) - F(r * r)), F(0.0))) * t)
    high = F(rho * t)
    return scale, offset, tail, mid, high


def words(blk, off, n):
    return struct.unpack_from(f"<{n}Q", bytes(blk[off: off + 8 * n]))


def full_scores_block(blk, plan: Plan, depth, w_s4):
    """All-stage score per live slot (no pruning): stages of src/scan.rs:453-634 with tau=-inf."""
    tomb = struct.unpack_from("<Q", bytes(blk[16:24]))[0]
    s0, s1, s2, s3, s4, s5 = (words(blk, o, n) for o, n in
                              ((512, 64), (1024, 128), (2048, 64), (2560, 64), (3072, 64), (3584, 64)))
    out = {}
    for v in range(64):
        if (tomb >> v) & 1:
            continue
        scale, offset, tail, mid, high = decode_meta(blk, v)
        if depth == 0:
            cd = F(0.0)
            for d in range(64):
                w = plan.bw3[d]
                if w != 0 and (s0[d] >> v) & 1:
                    cd = F(cd + w)
            out[v] = F(F(cd * scale) + F(offset * plan.prefix_sum))
            continue
        acc = F(0.0)
        for d in range(64):
            w = F(plan.eden_q_rot[d] * plan.eden_inv_sqrt_d) if plan.prefix_codec == 1 else plan.prefix[d]
            if w == 0:
                continue
            lv = ((s5[d] >> v) & 1) | (((s3[d] >> v) & 1) << 1) | (((s2[d] >> v) & 1) << 2) | (((s0[d] >> v) & 1) << 3)
            acc = F(acc + F((B4[lv] if plan.prefix_codec == 1 else F(lv)) * w))
        mid_n = max(mid, F(1e-6))
        high_n = max(high, F(0.0))
        if plan.prefix_codec == 1:
            score = F(plan.eden_mean_ip + F(scale * acc))
        else:
            score = F(F(acc * scale) + F(offset * plan.prefix_sum))
        s = plan.base
        for d in range(128):
            if (s1[d] >> v) & 1:
                s = F(s + plan.w2[d])
        score = F(score + F(s * mid_n))
        if depth == 2 and plan.has_tail_fold:
            t = plan.tbase
            for d in range(64):
                if (s4[d] >> v) & 1:
                    t = F(t + plan.tw2[d])
            score = F(score + F(F(t * max(high_n, F(1e-6))) * F(w_s4)))
        out[v] = score
    return out


def splitmix64(x):
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def ih_gauss(seed, idx):
    s = 0
    for j in range(3):
        h = splitmix64(((seed * 0xD1B54A32D192ED03) & M64) + idx * 3 + j & M64)
        s += (h & 0xFFFF) + ((h >> 16) & 0xFFFF) + ((h >> 32) & 0xFFFF) + (h >> 48)
    return F(F(2 * s + 12 - 786432) * F(1.0 / 131072.0))


def synth_row(seed, row, dims):
    x = [F(ih_gauss(seed, row * dims + d) * F(F(1.0) / np.sqrt(F(d + 1)))) for d in range(dims)]
    ss = F(0.0)
    for v in x:
        ss = F(ss + F(v * v))
    n = max(np.sqrt(ss), F(1e-12))
    return [F(v / n) for v in x]
