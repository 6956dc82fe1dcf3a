"""Pure-Python restatement of rustwood's CPU trainer for tiny inputs (test infrastructure).

An independent second restatement of src/cpu.rs:17-325 (and data.rs:86-146,
booster.rs:582-601), written with plain Python loops so the C oracle can be checked
against it bit-for-bit and golden fixtures can be generated from it. Both modes:
  exact=False: cpu.rs as written -- f32 chunked histograms combined by rayon's midpoint
               reduce tree, f64 gains and leaf sums, glibc expf;
  exact=True:  the fixed-point variant the GPU implements (see rw_expf.h): 17-bit
               histogram values, leaf sums of the unquantised g/h in a wide fixed point.
Only for n <= a few hundred rows: every operation is a Python-level scalar op.
"""
from __future__ import annotations

import ctypes
import math
import struct

import numpy as np

_libm = ctypes.CDLL("libm.so.6")
_libm.expf.argtypes = [ctypes.c_float]
_libm.expf.restype = ctypes.c_float

F32 = np.float32
QBITS = 17  # RW_QBITS in rustwood_b200/csrc/rw_expf.h


def f32(v) -> np.float32:
    return np.float32(v)


def glibc_expf(x: np.float32) -> np.float32:
    return F32(_libm.expf(float(x)))


def rw_expf(x: np.float32) -> np.float32:
    """Cody-Waite reduction + 12th-order Taylor series in double, rounded once."""
    xf = float(x)
    if xf != xf:
        return F32(x)
    if x > F32(89.0):
        return F32(np.inf)
    if x < F32(-104.0):
        return F32(0.0)
    ln2_hi = float.fromhex("0x1.62e42fee00000p-1")
    ln2_lo = float.fromhex("0x1.a39ef35793c76p-33")
    kd = float(round(xf * 1.4426950408889634))  # round-half-even == rint
    r = (xf + -(kd * ln2_hi)) + -(kd * ln2_lo)
    coef = [1.0 / math.factorial(i) for i in range(13)]
    p = coef[12]
    for i in range(11, -1, -1):
        p = p * r + coef[i]
    y = p * math.ldexp(1.0, int(kd))
    with np.errstate(over="ignore"):
        return F32(y)


def logistic_grad(p: np.float32, y: np.float32, exact: bool):
    e = rw_expf(F32(-p)) if exact else glibc_expf(F32(-p))
    pr = F32(F32(1.0) / F32(F32(1.0) + e))
    g = F32(pr - y)
    hv = F32(pr * F32(F32(1.0) - pr))
    return g, (hv if hv > F32(1e-6) else F32(1e-6))


def qscale_exp(m: np.float32) -> int:
    bits = struct.unpack("<I", struct.pack("<f", float(m)))[0]
    if bits & 0x7FFFFFFF == 0:
        return 0
    biased = (bits >> 23) & 0xFF
    e = QBITS - ((1 if biased == 0 else biased) - 126)
    return max(-126, min(100, e))


def quantize(x: np.float32, e: int) -> int:
    v = F32(x) * F32(2.0 ** e)
    return int(np.rint(v))


def wscale_exp(m: np.float32, n_rows: int) -> int:
    """Wide leaf-sum scale: (62 - bitlen(n)) - E with 2^(E-1) <= m < 2^E."""
    if m == 0:
        return 0
    _, e = math.frexp(float(m))  # m = f * 2^e with 0.5 <= f < 1
    return (62 - max(int(n_rows).bit_length(), 1)) - e


def wquantize(x: np.float32, w: int) -> int:
    return round(math.ldexp(float(x), w))  # exact product, round-half-even


def partition_point(cuts, v) -> int:
    lo, hi = 0, len(cuts)
    while lo < hi:
        mid = (lo + hi) // 2
        if cuts[mid] < v:
            lo = mid + 1
        else:
            hi = mid
    return lo


def boundaries(x: np.ndarray, n_bins: int, sample: int = 200_000, unique: bool = False):
    n, nf = x.shape
    nb1 = n_bins - 1
    stride = max(n // max(sample, 1), 1)
    out = []
    for f in range(nf):
        s = sorted([x[i, f] for i in range(0, n, stride)])  # stable
        m = len(s)
        if unique:
            u = []
            for v in s:
                if not u or u[-1] != v:
                    u.append(v)
            cand = [F32(F32(0.5) * F32(u[i] + u[i + 1])) for i in range(len(u) - 1)]
            for j in range(nb1):
                if not cand:
                    out.append(F32(np.inf))
                elif len(cand) <= nb1:
                    out.append(cand[j] if j < len(cand) else F32(np.inf))
                else:
                    pos = ((j + 1) * len(cand)) // (nb1 + 1)
                    out.append(cand[min(pos, len(cand) - 1)])
        else:
            b = []
            for j in range(nb1):
                q = (j + 1) / n_bins
                posd = q * (m - 1)
                pos = int(math.floor(posd + 0.5))  # f64::round, non-negative
                b.append(s[min(pos, m - 1)])
            for j in range(1, nb1):
                if b[j] <= b[j - 1]:
                    b[j] = b[j - 1]
            out.extend(b)
    return np.array(out, dtype=np.float32)


def _rayon_tree(vecs, lo, hi, zero):
    if hi - lo == 1:
        return [zero + v for v in vecs[lo]]
    mid = (hi - lo) // 2
    a = _rayon_tree(vecs, lo, lo + mid, zero)
    b = _rayon_tree(vecs, lo + mid, hi, zero)
    return [p + q for p, q in zip(a, b)]


def train(x, y, cuts, base, *, n_trees, depth, n_bins, learning_rate=0.1, lambda_=1.0,
          min_child_h=1e-3, objective="logistic", subtract=True, exact=True, n_threads=1,
          subsample=1.0, pgbm=False):
    n, nf = x.shape
    nb1 = n_bins - 1
    leaves = 1 << depth
    lam, lr, mc = float(F32(lambda_)), float(F32(learning_rate)), float(F32(min_child_h))
    bins = [[partition_point(cuts[f * nb1:(f + 1) * nb1], x[r, f]) for f in range(nf)]
            for r in range(n)]
    pred = [F32(base)] * n
    feat, thr, thr_bin = [], [], []
    leafval = [F32(0)] * (n_trees * leaves)
    leafvar = [F32(0)] * (n_trees * leaves)  # PGBM (exact mode)
    fi_gain = [F32(0)] * nf
    fi_count = [F32(0)] * nf
    stride = 1
    if F32(subsample) < F32(0.999):
        stride = max(int(math.floor(1.0 / float(F32(subsample)) + 0.5)), 1)
    for t in range(n_trees):
        g, h = [F32(0)] * n, [F32(1)] * n
        for i in range(n):
            if objective == "logistic":
                g[i], h[i] = logistic_grad(pred[i], F32(y[i]), exact)
            else:
                g[i], h[i] = F32(pred[i] - F32(y[i])), F32(1)
        samp = list(range(t % stride, n, stride)) if stride > 1 else list(range(n))
        node = [0] * n
        if exact:
            mg = max([abs(g[r]) for r in samp] + [F32(0)])
            mh = max([h[r] for r in samp] + [F32(0)])
            eg, eh = qscale_exp(mg), qscale_exp(mh)
            wg, wh = wscale_exp(mg, n), wscale_exp(mh, n)
            qg = {r: quantize(g[r], eg) for r in samp}
            qh = {r: quantize(h[r], eh) for r in samp}
            inv_g, inv_h = 2.0 ** -eg, 2.0 ** -eh
        prev = None
        for level in range(depth):
            nn = 1 << level

            def build(index_nodes, odd_only):
                size = index_nodes * nf * n_bins * 2
                if exact:
                    hist = [0] * size
                    for r in samp:
                        nv = node[r]
                        if odd_only:
                            if nv & 1 == 0:
                                continue
                            nv >>= 1
                        for f in range(nf):
                            idx = ((nv * nf + f) * n_bins + bins[r][f]) * 2
                            hist[idx] += qg[r]
                            hist[idx + 1] += qh[r]
                    return hist
                m = len(samp)
                chunk = -(-m // n_threads)
                locs = []
                for ti in range(n_threads):
                    loc = [F32(0)] * size
                    for q in range(ti * chunk, min((ti + 1) * chunk, m)):
                        r = samp[q]
                        nv = node[r]
                        if odd_only:
                            if nv & 1 == 0:
                                continue
                            nv >>= 1
                        for f in range(nf):
                            idx = ((nv * nf + f) * n_bins + bins[r][f]) * 2
                            loc[idx] = F32(loc[idx] + g[r])
                            loc[idx + 1] = F32(loc[idx + 1] + h[r])
                    locs.append(loc)
                return _rayon_tree(locs, 0, n_threads, F32(0))

            if level == 0 or not subtract:
                hist = build(nn, False)
            else:
                odd = build(nn // 2, True)
                sl = nf * n_bins * 2
                hist = [0] * (nn * sl)
                for i in range(nn // 2):
                    for k in range(sl):
                        hist[(2 * i + 1) * sl + k] = odd[i * sl + k]
                        hist[(2 * i) * sl + k] = (prev[i * sl + k] - odd[i * sl + k]) if exact \
                            else F32(prev[i * sl + k] - odd[i * sl + k])
            best = (-math.inf, 0, 0)
            for f in range(nf):
                gain = [0.0] * nb1
                for nd in range(nn):
                    hb = (nd * nf + f) * n_bins
                    pg, ph = [], []
                    if exact:
                        sg = sh = 0
                        for b in range(n_bins):
                            sg += hist[(hb + b) * 2]
                            sh += hist[(hb + b) * 2 + 1]
                            pg.append(float(sg) * inv_g)
                            ph.append(float(sh) * inv_h)
                    else:
                        gl = hl = 0.0
                        for b in range(n_bins):
                            gl += float(hist[(hb + b) * 2])
                            hl += float(hist[(hb + b) * 2 + 1])
                            pg.append(gl)
                            ph.append(hl)
                    gt, ht = pg[-1], ph[-1]
                    parent = gt * gt / (ht + lam)
                    for b in range(nb1):
                        gl, hl = pg[b], ph[b]
                        gr, hr = gt - gl, ht - hl
                        valid = 1.0 if (hl >= mc and hr >= mc) else 0.0
                        gain[b] += valid * (gl * gl / (hl + lam) + gr * gr / (hr + lam) - parent)
                bg, bb = -math.inf, 0
                for b, gv in enumerate(gain):
                    if gv > bg:
                        bg, bb = gv, b
                if bg > best[0]:
                    best = (bg, f, bb)
            bg, bf, bb = best
            feat.append(bf)
            thr.append(cuts[bf * nb1 + bb])
            thr_bin.append(bb)
            fi_gain[bf] = F32(fi_gain[bf] + F32(max(bg, 0.0)))
            fi_count[bf] = F32(fi_count[bf] + F32(1))
            for r in range(n):
                node[r] = node[r] * 2 + (1 if bins[r][bf] > bb else 0)
            prev = hist
        if exact:
            # exact integer sums of the unquantised g/h in the wide fixed point
            sg, sh = [0] * leaves, [0] * leaves
            for r in samp:
                sg[node[r]] += wquantize(g[r], wg)
                sh[node[r]] += wquantize(h[r], wh)
            lg = [math.ldexp(float(v), -wg) for v in sg]
            lc = [math.ldexp(float(v), -wh) for v in sh]
            if pgbm:
                # gpu_kernels.rs:1015-1080: per-leaf sum of g*g (f32 products); the wide
                # scale comes from (max |g|)^2 in f32, which bounds every product
                m2 = F32(mg * mg)
                if not np.isfinite(m2):
                    m2 = np.finfo(np.float32).max
                w2 = wscale_exp(m2, n)
                s2 = [0] * leaves
                for r in samp:
                    s2[node[r]] += wquantize(F32(g[r] * g[r]), w2)
                for l in range(leaves):
                    G, H, S2 = lg[l], lc[l], math.ldexp(float(s2[l]), -w2)
                    if H > 1.0:
                        m = G / H
                        v = S2 / H - m * m
                        leafvar[t * leaves + l] = F32(lr * lr * (v if v > 0.0 else 0.0))
        else:
            m = len(samp)
            chunk = -(-m // n_threads)
            lgs, lcs = [], []
            for ti in range(n_threads):
                a, c = [0.0] * leaves, [0.0] * leaves
                for q in range(ti * chunk, min((ti + 1) * chunk, m)):
                    r = samp[q]
                    a[node[r]] += float(g[r])
                    c[node[r]] += float(h[r])
                lgs.append(a)
                lcs.append(c)
            lg = _rayon_tree(lgs, 0, n_threads, 0.0)
            lc = _rayon_tree(lcs, 0, n_threads, 0.0)
        for l in range(leaves):
            leafval[t * leaves + l] = F32(-lr * lg[l] / (lc[l] + lam))
        for r in range(n):
            pred[r] = F32(pred[r] + leafval[t * leaves + node[r]])
    return dict(feat=np.array(feat, np.uint32), thr=np.array(thr, np.float32),
                thr_bin=np.array(thr_bin, np.uint32), leafval=np.array(leafval, np.float32),
                leafvar=np.array(leafvar, np.float32),
                fi_gain=np.array(fi_gain, np.float32), fi_count=np.array(fi_count, np.float32))


def predict(x, feat, thr, leafval, base, n_trees, depth):
    out = []
    nl = 1 << depth
    for row in x:
        acc = F32(base)
        for t in range(n_trees):
            leaf = 0
            for d in range(depth):
                k = t * depth + d
                leaf = leaf * 2 + (1 if row[feat[k]] > thr[k] else 0)
            acc = F32(acc + leafval[t * nl + leaf])
        out.append(acc)
    return np.array(out, np.float32)
