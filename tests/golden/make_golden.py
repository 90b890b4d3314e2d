#!/usr/bin/env python3
"""Write the golden vectors in tests/golden/ by running the reference itself.

Imports the reference's own glint_np.py, glint_codec.py and glint_htile_sim.py
(Jadon-Fox/glint) from a read-only checkout given by --ref (default: the
GLINT_REFERENCE environment variable) and records, for seeded inputs:

  tables.json           PARENT and CELLS as f32 bit patterns (glint_codec.py:11-28, 92-113)
  encode_bf16.npz       glint_np.encode_f32(glint_np.dense_to_f32("BF16", ...), bs)
                        for the BF16 cases (glint_np.py:16-24, 63-83)
  encode_f32.npz        glint_np.encode_f32 on f32 inputs: ties, midpoints, ulp
                        neighbours, +-0, NaN, +-inf, denormals (glint_np.py:41-83)
  expand.npz            glint_np.expand and glint_np.f32_to_bf16_bytes
                        (glint_np.py:25-31, 84-92) over all 256 codes and special
                        absmax values
  htile.npz             glint_htile_sim.htile_gemm_flat (glint_htile_sim.py:22-50)
                        on small shapes, K tails and blocksize 23

The fixtures are committed, so the tests never need the reference at run time.
Run:  python tests/golden/make_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def synth_bf16(rng: np.random.Generator, n: int, outlier_frac: float = 0.001) -> np.ndarray:
    """N(0, 0.02) with floor(frac*n) entries x20, rounded to BF16 (RNE) -> uint16 bits."""
    w = rng.normal(0.0, 0.02, n).astype(np.float32)
    k = int(outlier_frac * n)
    if k:
        idx = rng.choice(n, size=k, replace=False)
        w[idx] *= np.float32(20.0)
    u = w.view(np.uint32)
    return ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype(np.uint16)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GLINT_REFERENCE", ""))
    args = ap.parse_args()
    if not args.ref or not Path(args.ref, "glint_np.py").is_file():
        print("need --ref pointing at a Jadon-Fox/glint checkout", file=sys.stderr)
        return 2
    sys.path.insert(0, str(Path(args.ref).resolve()))
    import glint_codec  # noqa: E402
    import glint_htile_sim  # noqa: E402
    import glint_np as G  # noqa: E402

    # ---- tables
    tables = {
        "parent_bits": [int(x) for x in G.PARENT_F32.view(np.uint32)],
        "cells_bits": [int(x) for x in G.CELLS_F32.reshape(-1).view(np.uint32)],
    }
    (OUT / "tables.json").write_text(json.dumps(tables, indent=1) + "\n")

    rng = np.random.default_rng(0)

    # ---- BF16 encode cases
    cases = {}

    def add_bf16(name, bits, bs):
        bits = np.ascontiguousarray(bits, np.uint16)
        n = bits.size
        w = G.dense_to_f32("BF16", bits.tobytes(), n)
        h, p, am = G.encode_f32(w, bs)
        cases[name + "__w"] = bits
        cases[name + "__bs"] = np.array([bs], np.int64)
        cases[name + "__hole"] = np.frombuffer(h, np.uint8)
        cases[name + "__plug"] = np.frombuffer(p, np.uint8)
        cases[name + "__absmax"] = am.astype(np.float32)
        ex = G.expand(h, p, am, n, bs)
        cases[name + "__expand_f32"] = ex.astype(np.float32)
        cases[name + "__expand_bf16"] = np.frombuffer(G.f32_to_bf16_bytes(ex), np.uint16)

    add_bf16("llama_like", synth_bf16(rng, 64 * 1000), 64)
    add_bf16("toy_q", synth_bf16(rng, 16 * 64, 0.0), 64)
    add_bf16("odd_straddle", synth_bf16(rng, 7 * 63, 0.0), 64)
    zb = synth_bf16(rng, 4 * 128, 0.0)
    zb[:64] = 0
    add_bf16("zero_block", zb, 64)
    add_bf16("bs23", synth_bf16(rng, 999), 23)
    add_bf16("bs1", synth_bf16(rng, 37, 0.0), 1)
    add_bf16("bs128_odd", synth_bf16(rng, 128 * 9 + 5), 128)
    add_bf16("single", np.array([0x3F80], np.uint16), 64)
    add_bf16("gpu_ok_probe", np.array([0x3F80, 0x0000], np.uint16), 64)
    # BF16 specials: NaN, +-inf, -0, denormals, an all-NaN block, a block with inf,
    # a block of denormals only, the largest finite values.
    sp = synth_bf16(rng, 64 * 8, 0.0)
    sp[3] = 0x7FC0          # NaN
    sp[5] = 0xFFC1          # -NaN with payload
    sp[64:128] = 0x7FC0     # all-NaN block
    sp[130] = 0x7F80        # +inf in block 2
    sp[140] = 0xFF80        # -inf in block 2
    sp[192:256] = rng.integers(0, 0x80, 64, dtype=np.uint16) | (rng.integers(0, 2, 64, dtype=np.uint16) << 15)  # denormals
    sp[256] = 0x8000        # -0
    sp[320:384] = 0x8000    # block of -0 only
    sp[400] = 0x7F7F        # max finite
    sp[401] = 0xFF7F
    sp[448:512] = np.uint16(0x7F7F) - rng.integers(0, 4, 64, dtype=np.uint16)
    add_bf16("specials", sp, 64)
    # Every BF16 bit pattern once, in blocks of 64 (covers every exponent and NaN/inf).
    add_bf16("all_bf16", rng.permutation(np.arange(65536, dtype=np.uint32)).astype(np.uint16), 64)
    np.savez_compressed(OUT / "encode_bf16.npz", **cases)

    # ---- f32 encode cases: one weight of exactly 1.0 per block makes absmax 1 and
    # v == w, so the values below land exactly on the decision edges.
    f = G.CELLS_FLAT
    par = G.PARENT_F32
    mids = ((f[1:] + f[:-1]) / 2).astype(np.float32)
    pmid = ((par[1:] + par[:-1]) / 2).astype(np.float32)
    up = lambda a: np.nextafter(a, np.float32(2))  # noqa: E731
    dn = lambda a: np.nextafter(a, np.float32(-2))  # noqa: E731
    edge = np.concatenate([f, mids, pmid, par, up(mids), dn(mids), up(pmid), dn(pmid), up(f), dn(f),
                           np.float32([1, -1, 0, -0.0, np.nan, np.inf, -np.inf]),
                           rng.uniform(-1, 1, 4000).astype(np.float32)]).astype(np.float32)
    per = 63
    nb = (edge.size + per - 1) // per
    w = np.zeros(nb * 64, np.float32)
    for b in range(nb):
        chunk = edge[b * per:(b + 1) * per]
        w[b * 64] = 1.0
        w[b * 64 + 1:b * 64 + 1 + chunk.size] = chunk
    # the inf entries make their block's absmax inf; keep them, that is a case too
    f32cases = {}

    def add_f32(name, wf, bs):
        wf = np.ascontiguousarray(wf, np.float32)
        h, p, am = G.encode_f32(wf, bs)
        f32cases[name + "__w"] = wf
        f32cases[name + "__bs"] = np.array([bs], np.int64)
        f32cases[name + "__hole"] = np.frombuffer(h, np.uint8)
        f32cases[name + "__plug"] = np.frombuffer(p, np.uint8)
        f32cases[name + "__absmax"] = am.astype(np.float32)

    add_f32("edges", w, 64)
    add_f32("gauss_f32", rng.normal(0, 0.02, 3 * 64 * 10 + 1).astype(np.float32), 64)
    den = (rng.integers(1, 1 << 23, 640, dtype=np.uint32) | (rng.integers(0, 2, 640, dtype=np.uint32) << 31)).view(np.float32)
    add_f32("denormal_f32", den, 64)
    np.savez_compressed(OUT / "encode_f32.npz", **f32cases)

    # ---- expand over all 256 codes with special absmax values
    codes = np.arange(256 * 4, dtype=np.int64) % 256
    n = codes.size + 3  # odd n: pad nibble
    hh = np.concatenate([(codes >> 4), rng.integers(0, 16, 3)]).astype(np.uint8)
    pp = np.concatenate([(codes & 15), rng.integers(0, 16, 3)]).astype(np.uint8)
    hole_pk = G.pack_nibbles(hh)
    plug_pk = G.pack_nibbles(pp)
    bs = 16
    nam = (n + bs - 1) // bs
    am = np.abs(rng.normal(0, 0.05, nam)).astype(np.float32)
    am[1] = 0.0
    am[2] = np.float32(np.nan)
    am[3] = np.float32(np.inf)
    am[4] = np.float32(3.0e38)              # products overflow or round up to inf in BF16
    am[5] = np.float32(1e-40)               # denormal scale
    am[6] = np.float32(3.3895314e38)        # near the largest finite BF16
    am[7] = np.float32(1.0)
    ex = G.expand(hole_pk.tobytes(), plug_pk.tobytes(), am, n, bs)
    np.savez_compressed(OUT / "expand.npz", hole=hole_pk, plug=plug_pk, absmax=am, n=np.array([n]),
                        bs=np.array([bs]), expand_f32=ex.astype(np.float32),
                        expand_bf16=np.frombuffer(G.f32_to_bf16_bytes(ex), np.uint16))

    # ---- H-TILE on small shapes through the reference simulator (f64 sums)
    ht = {}
    shapes = [(4, 8, 64, 64), (7, 23, 64, 64), (3, 5, 70, 64), (2, 3, 199, 23), (1, 17, 128, 64),
              (16, 16, 32, 64), (5, 9, 1, 23)]
    for (M, N, K, bsz) in shapes:
        nW = N * K
        hb = synth_bf16(rng, nW)
        wv = G.dense_to_f32("BF16", hb.tobytes(), nW)
        h, p, amx = G.encode_f32(wv, bsz)
        xu = rng.normal(0, 1, M * K).astype(np.float32).view(np.uint32)  # N(0,1) activations, RNE to BF16
        xb = ((xu + (np.uint32(0x7FFF) + ((xu >> 16) & np.uint32(1)))) >> 16).astype(np.uint16)
        xf = G.dense_to_f32("BF16", xb.tobytes(), M * K)
        hi = list(G.unpack_nibbles(h, nW))
        pi = list(G.unpack_nibbles(p, nW))
        y = glint_htile_sim.htile_gemm_flat([float(v) for v in xf], hi, pi, [float(a) for a in amx],
                                            M, N, K, bsz, 64, False)
        key = f"m{M}_n{N}_k{K}_bs{bsz}"
        ht[key + "__hole"] = np.frombuffer(h, np.uint8)
        ht[key + "__plug"] = np.frombuffer(p, np.uint8)
        ht[key + "__absmax"] = amx.astype(np.float32)
        ht[key + "__x"] = xb
        ht[key + "__y"] = np.array(y, np.float64)
        ht[key + "__shape"] = np.array([M, N, K, bsz], np.int64)
    np.savez_compressed(OUT / "htile.npz", **ht)
    assert glint_codec.CELLS  # imported for the tables' provenance
    print("golden vectors written to", OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
