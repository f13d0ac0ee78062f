"""Generate the golden fixtures tests/golden/{paris,bunny}.npz from the reference's data files.

    python tests/golden/make_fixtures.py <REFERENCE_ROOT>

The reference ships, for its website, the factorization PATHPACK.jl computed with mlu(MinPlus(), A) in
Float32 for two demo graphs (docs/src/public/data/<name>-lu.bin.gz, written by docs/site_factors.jl:136-205)
and the demo graphs themselves (<name>.bin.gz).  This script rebuilds each graph exactly as
docs/site_factors.jl:44-104 specifies (Paris: weights wm/1000 in Float32; bunny: Float32 coordinates and
V8's Math.hypot, both arcs per edge, parallel arcs combined with min) and stores, 0-based:
  - the arcs (I, J, W) of A,
  - the reference's symbolic structure (Rptr, Sptr, Stgt, Bptr, Fptr, Nptr, Ntgt, perm = rperm),
  - the reference's factor values: D (upper triangle and diagonal of UDval, strict lower triangle of LDval),
    UL (ULval) and LL (LLval).
The file format (bin.ts: uint32 header length, JSON header {meta, arrays: name => [dtype, offset, count]},
4-byte aligned arrays, gzip) is docs/site_factors.jl:23-35 / :119-134.
"""
import gzip
import json
import math
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TYPES = {"uint8": np.uint8, "uint16": np.uint16, "uint32": np.uint32, "int16": np.int16, "int32": np.int32,
         "float32": np.float32}


def readbin(path):
    raw = gzip.open(path).read()
    hl = struct.unpack("<I", raw[:4])[0]
    head = json.loads(raw[4:4 + hl])
    base = 4 + hl
    arrays = {}
    for k, (t, off, cnt) in head["arrays"].items():
        T = TYPES[t]
        arrays[k] = np.frombuffer(raw, dtype=T, count=cnt, offset=base + off).copy()
    return head["meta"], arrays


def jshypot(*xs):
    """Math.hypot as V8 computes it (docs/site_factors.jl:79-98): scale by the largest magnitude, Kahan sum."""
    mx = 0.0
    for x in xs:
        mx = max(mx, abs(x))
    if mx == 0:
        return 0.0
    s = 0.0
    comp = 0.0
    for x in xs:
        r = abs(x) / mx
        t = r * r - comp
        prel = s + t
        comp = (prel - s) - t
        s = prel
    return math.sqrt(s) * mx


def paris(data):
    meta, a = readbin(os.path.join(data, "paris.bin.gz"))
    n, m = int(meta["n"]), int(meta["m"])
    I = a["ei"].astype(np.int64)
    J = a["ej"].astype(np.int64)
    W = np.array([np.float32(float(w) / 1000) for w in a["wm"]], dtype=np.float32)
    assert len(I) == len(J) == m
    return n, I, J, W


def bunny(data):
    meta, a = readbin(os.path.join(data, "bunny.bin.gz"))
    n, nf = int(meta["n"]), int(meta["f"])
    lo, scale = meta["lo"], float(meta["scale"])
    pos, tri = a["pos"], a["tri"]
    P = np.array([np.float32(lo[i % 3] + float(pos[i]) / scale) for i in range(3 * n)], dtype=np.float32)
    seen, I, J, W = set(), [], [], []
    for f in range(nf):
        i, j, k = int(tri[3 * f]), int(tri[3 * f + 1]), int(tri[3 * f + 2])
        for p, q in ((i, j), (j, k), (k, i)):
            key = min(p, q) * 65536 + max(p, q)
            if key in seen:
                continue
            seen.add(key)
            dx = float(P[3 * p]) - float(P[3 * q])
            dy = float(P[3 * p + 1]) - float(P[3 * q + 1])
            dz = float(P[3 * p + 2]) - float(P[3 * q + 2])
            I.append(p)
            J.append(q)
            W.append(np.float32(jshypot(dx, dy, dz)))
    return n, np.array(I, np.int64), np.array(J, np.int64), np.array(W, np.float32)


def symmetric_min(n, I, J, W):
    """sparse(vcat(I, J), vcat(J, I), vcat(W, W), n, n, min) as sorted unique arcs."""
    ii = np.concatenate([I, J])
    jj = np.concatenate([J, I])
    ww = np.concatenate([W, W])
    key = jj * n + ii
    order = np.lexsort((ww, key))
    key, ii, jj, ww = key[order], ii[order], jj[order], ww[order]
    first = np.ones(len(key), bool)
    first[1:] = key[1:] != key[:-1]
    return ii[first], jj[first], ww[first]


def factorfile(data, name, n):
    meta, a = readbin(os.path.join(data, name + "-lu.bin.gz"))
    assert meta["n"] == n and meta["semiring"] == "MinPlus" and meta["eltype"] == "Float32"
    g = lambda k: a[k].astype(np.int64)
    return dict(
        Rptr=g("Rptr") - 1, Sptr=g("Sptr") - 1, Stgt=g("Stgt") - 1, Bptr=g("Bptr") - 1, Fptr=g("Fptr") - 1,
        Nptr=g("Nptr") - 1, Ntgt=g("Ntgt") - 1, perm=g("rperm") - 1, cinvp=g("cinvp") - 1,
        D=a["D"].astype(np.float32), UL=a["UL"].astype(np.float32), LL=a["LL"].astype(np.float32),
        Nval=a["Nval"].astype(np.float32))


def main(root):
    data = os.path.join(root, "docs", "src", "public", "data")
    for name, make in (("paris", paris), ("bunny", bunny)):
        n, I, J, W = make(data)
        Ia, Ja, Wa = symmetric_min(n, I, J, W)
        F = factorfile(data, name, n)
        assert np.array_equal(F["perm"][F["cinvp"]], np.arange(n))
        out = os.path.join(HERE, name + ".npz")
        np.savez_compressed(out, n=n, I=Ia.astype(np.int32), J=Ja.astype(np.int32), W=Wa,
                            **{k: v.astype(np.int32) if v.dtype == np.int64 else v for k, v in F.items() if k != "cinvp"})
        print("%s: n=%d arcs=%d fronts=%d -> %s (%.0f kB)" % (name, n, len(Ia), len(F["Rptr"]) - 1, out,
                                                            os.path.getsize(out) / 1e3))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_fixtures.py <path of a PATHPACK.jl checkout>")
    main(sys.argv[1])
