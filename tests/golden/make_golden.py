"""Generates the golden fixtures in tests/golden/ (run from the repo root):

    python tests/golden/make_golden.py

The reference (Rust) cannot be built or run here, so the fixtures come from
implementations that share no code with the C oracle:
  * quantize / dequantize: the vectorised numpy restatement in
    oracle/quant_numpy.py of crates/kvforge-cpu/src/quantize.rs;
  * rANS container: the pure-Python encoder below, written from the container
    specification (kvforge_b200/csrc/kvf_rans.cu header comment);
  * ranks: numpy's fp64 SVD + a Python restatement of select_rank
    (crates/kvforge-cpu/src/projection.rs:31-59).
The reference's own known-answer values (quantize.rs:246-258,
projection.rs:242-253, entropy.rs:192-199) are stored alongside.
"""
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))
from oracle import quant_numpy as QN  # noqa: E402

PROB_BITS = 13
M = 1 << PROB_BITS
L = 1 << 16


def py_normalize(freq):
    N = int(sum(freq))
    q = [0 if f == 0 else max(1, (f * M) // N) for f in freq]
    S = sum(q)
    argmax = 0
    for s in range(256):
        if freq[s] > freq[argmax]:
            argmax = s
    if S < M:
        q[argmax] += M - S
    while S > M:
        best = -1
        for s in range(256):
            if q[s] > 1 and (best < 0 or q[s] > q[best]):
                best = s
        d = min(S - M, q[best] - 1)
        q[best] -= d
        S -= d
    cum, c = [], 0
    for s in range(256):
        cum.append(c)
        c += q[s]
    return q, cum


def py_rans_encode(data: bytes, chunk: int) -> bytes:
    n = len(data)
    freq = [0] * 256
    for b in data:
        freq[b] += 1
    q, cum = py_normalize(freq)
    nc = (n + chunk - 1) // chunk
    payloads = []
    for c in range(nc):
        sym = data[c * chunk:(c + 1) * chunk]
        steps = (len(sym) + 31) // 32
        states, streams = [], []
        for lane in range(32):
            x = L
            emitted = []  # in emission order
            for st in range(steps - 1, -1, -1):
                i = st * 32 + lane
                if i >= len(sym):
                    continue
                s = sym[i]
                f = q[s]
                if x >= (f << (32 - PROB_BITS)):
                    emitted.append(x & 0xFFFF)
                    x >>= 16
                x = ((x // f) << PROB_BITS) + (x % f) + cum[s]
            states.append(x)
            streams.append(list(reversed(emitted)))  # the decoder reads the last emitted word first
        words = [w for stream in streams for w in stream]
        body = (struct.pack("<32I", *states) + struct.pack("<32H", *[len(t) for t in streams])
                + struct.pack(f"<{len(words)}H", *words))
        if len(words) % 2:
            body += b"\x00\x00"
        payloads.append(body)
    hdr_len = 32 + 4 * (nc + 1)
    offs, pos = [], hdr_len
    for p in payloads:
        offs.append(pos)
        pos += len(p)
    offs.append(pos)
    header = struct.pack("<IIIIQII", 0x3252564B, PROB_BITS, 32, chunk, n, nc, hdr_len)
    return header + struct.pack(f"<{nc + 1}I", *offs) + b"".join(payloads), np.array(freq, np.uint32)


def py_select_rank(sv, threshold, max_rank=None):
    sv = [float(np.float32(s)) for s in sv]
    if not sv:
        return 0
    total = sum(s * s for s in sv)
    if total < 1e-12:
        return 1
    cum, rank = 0.0, 0
    for s in sv:
        cum += s * s
        rank += 1
        if cum / total >= threshold:
            break
    if max_rank:
        rank = min(rank, max_rank)
    return max(rank, 1)


def quant_cases(rng):
    cases = {}
    shapes = [(2, 9, 8), (3, 5, 7), (1, 64, 32), (2, 3, 1), (4, 33, 12)]
    for si, shp in enumerate(shapes):
        x = rng.uniform(-1, 1, shp).astype(np.float32)
        if si == 0:
            x[0, :, 3] = 0.25          # constant column -> scale 1.0
            x[1, 4, :] = 0.0           # zero row
            x[1, 5, 2] = -0.0
            x[0, 2, 5] = np.float32(1e-3)
        if si == 4:
            x[2, 7, 3] = np.nan        # NaN ignored by min/max, coded 0
            x[3, 1, 1] = np.inf
            x[3, 2, 2] = -np.inf
        for dt in (QN.INT4, QN.INT8):
            for ax in (QN.PER_CHANNEL, QN.PER_TOKEN):
                p, s, m = QN.quantize(x, dt, ax)
                d = QN.dequantize(p, s, m, dt, ax, shp)
                key = f"q{si}_{dt}_{ax}"
                cases[key + "_x"] = x
                cases[key + "_packed"] = p
                cases[key + "_scales"] = s
                cases[key + "_mins"] = m
                cases[key + "_deq"] = d
    return cases


def rans_cases(rng):
    cases = {}
    inputs = {
        "uniform256": (np.arange(256, dtype=np.uint8), 16384),
        "skewed1000": (np.concatenate([np.zeros(100, np.uint8), [1], np.zeros(99, np.uint8), [2],
                                       np.zeros(99, np.uint8), [255], np.zeros(699, np.uint8)]).astype(np.uint8), 16384),
        "nibbles_multi": (rng.integers(0, 16, 1000).astype(np.uint8) | (rng.integers(0, 4, 1000).astype(np.uint8) << 4), 96),
        "single": (np.full(77, 9, np.uint8), 64),
        "tail33": (rng.integers(0, 256, 33).astype(np.uint8), 32),
        "gauss": (np.clip(np.round(rng.normal(128, 12, 5000)), 0, 255).astype(np.uint8), 1024),
    }
    for name, (data, chunk) in inputs.items():
        comp, freq = py_rans_encode(bytes(data.tobytes()), chunk)
        cases[f"r_{name}_data"] = data
        cases[f"r_{name}_chunk"] = np.array([chunk], np.uint32)
        cases[f"r_{name}_comp"] = np.frombuffer(comp, np.uint8)
        cases[f"r_{name}_freq"] = freq
    return cases


def rank_cases(rng):
    cases = {}
    x = np.zeros((3, 200, 16), np.float32)
    for h in range(3):
        U = rng.standard_normal((200, 6))
        V = np.linalg.qr(rng.standard_normal((16, 6)))[0].T
        s = 0.7 ** np.arange(6) * (h + 1)
        x[h] = (U * s) @ V + 0.05 * rng.standard_normal((200, 16))
    cases["p_x"] = x
    for thr in (0.5, 0.75, 0.9, 0.99):
        ranks = []
        for h in range(3):
            sv = np.linalg.svd(x[h].astype(np.float64), compute_uv=False)
            ranks.append(py_select_rank(sv, thr))
        cases[f"p_ranks_{int(thr * 100)}"] = np.array(ranks, np.uint64)
    return cases


def main():
    rng = np.random.default_rng(20260101)
    out = {}
    out.update(quant_cases(rng))
    out.update(rans_cases(rng))
    out.update(rank_cases(rng))
    # reference known answers
    out["kat_pack_3_12"] = np.array([0xC3], np.uint8)            # quantize.rs:247
    out["kat_select_rank_sv"] = np.array([10, 5, 2, 1, 0.5], np.float32)
    out["kat_select_rank_expect"] = np.array([2, 2, 1], np.uint64)  # projection.rs:246-252
    out["kat_hist_data"] = np.array([0, 0, 0, 1, 1, 2], np.uint8)
    out["kat_hist_expect"] = np.array([3, 2, 1, 0], np.uint32)     # entropy.rs:195-198
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
