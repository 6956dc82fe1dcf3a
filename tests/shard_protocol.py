"""Row-sharded exact training, one rank per shard (test infrastructure).

A numpy restatement of the exchange protocol that librwgpu runs over NCCL when a
context is created with world > 1 (rw_fit_dataset in rwgpu.cu), driven here over any
torch.distributed backend so the protocol itself can be checked on CPU ranks (gloo):

  per tree   gradients on the local rows; the sampled set uses the GLOBAL row id
             (row_offset + i) for stride subsampling and for the GOSS keep hash;
             GOSS: the k-th largest |g| over all ranks by a 4-pass MSB-first radix select
             on the f32 bit patterns, one all-reduce(sum) of 256 digit counts per pass;
             fixed-point scales: one all-reduce(max) of the f32 bit patterns of
             max|g| and max h over the sampled rows;
  per level  local int64 histogram of the odd children (all nodes at level 0 or without
             subtraction), one all-reduce(sum) of it, even = parent - odd locally, then the
             same split scan on every rank (identical splits, nothing broadcast);
  leaves     one all-reduce(sum) of the per-leaf integer sums (wide fixed point of the
             unquantised g/h, scaled by the global row count).

Every all-reduce is of integers, so the model is bit-identical to the single-process
exact trainer at any rank count (src/cpu.rs:123-325 with exact accumulation). Only
tests import this module.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
QBITS = 17  # RW_QBITS in rustwood_b200/csrc/rw_expf.h
GOSS_SALT = np.uint64(0x00424552455A4B41)


def qscale_exp(max_bits: int) -> int:
    """Exponent e such that max * 2^e < 2^QBITS (rw_qscale_exp in rw_expf.h)."""
    if max_bits & 0x7FFFFFFF == 0:
        return 0
    biased = (max_bits >> 23) & 0xFF
    e = QBITS - ((1 if biased == 0 else biased) - 126)
    return max(-126, min(100, e))


def quantize(x: np.ndarray, e: int) -> np.ndarray:
    """round-half-even(f32(x) * f32(2^e)) as int64 (rw_quantize)."""
    return np.rint(x.astype(F32) * F32(2.0 ** e)).astype(np.int64)


def wscale_exp(max_bits: int, n_rows: int) -> int:
    """Wide leaf-sum exponent (62 - bitlen(n)) - E, 2^(E-1) <= max < 2^E (rw_wscale_exp)."""
    if max_bits & 0x7FFFFFFF == 0:
        return 0
    biased = (max_bits >> 23) & 0xFF
    return (62 - max(int(n_rows).bit_length(), 1)) - ((1 if biased == 0 else biased) - 126)


def wquantize(x: np.ndarray, w: int) -> np.ndarray:
    """round-half-even(f64(x) * 2^w) as int64 (rw_wquantize); the product is exact."""
    return np.rint(x.astype(np.float64) * 2.0 ** w).astype(np.int64)


def f32_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, F32).view(np.uint32).astype(np.int64)


class Exchange:
    """The three collectives the protocol needs, over torch.distributed (or none)."""

    def __init__(self, dist=None):
        self.dist = dist

    def _reduce(self, a: np.ndarray, op) -> np.ndarray:
        if self.dist is None:
            return a
        import torch
        t = torch.from_numpy(np.ascontiguousarray(a, np.int64).copy())
        self.dist.all_reduce(t, op=op)
        return t.numpy()

    def sum(self, a: np.ndarray) -> np.ndarray:
        return self._reduce(a, None if self.dist is None else self.dist.ReduceOp.SUM)

    def max(self, a: np.ndarray) -> np.ndarray:
        return self._reduce(a, None if self.dist is None else self.dist.ReduceOp.MAX)


def kth_largest_abs_bits(g: np.ndarray, k: int, ex: Exchange) -> int:
    """Bit pattern of the k-th (0-based) largest |g| over all ranks: MSB-first radix
    select over the 4 bytes of the f32 bit pattern (non-negative floats order like
    their bits), one all-reduce of 256 counts per byte."""
    bits = f32_bits(np.abs(g))
    prefix, mask = 0, 0
    for shift in (24, 16, 8, 0):
        cand = bits[(bits & mask) == prefix]
        counts = np.bincount((cand >> shift) & 0xFF, minlength=256).astype(np.int64)
        counts = ex.sum(counts)
        acc = 0
        for digit in range(255, -1, -1):  # descending: largest values first
            if acc + counts[digit] > k:
                break
            acc += counts[digit]
        k -= acc
        prefix |= digit << shift
        mask |= 0xFF << shift
    return prefix


def goss_select(g, h, gid, n_global, top, other, tree, ex):
    """src/cpu.rs:64-110 over sharded rows: returns (sampled mask, g, h)."""
    tn = top * n_global
    topn = min(max(int(tn) if tn > 0 else 0, 1), n_global)
    k = min(topn - 1, n_global - 1)
    thresh = np.array([kth_largest_abs_bits(g, k, ex)], np.uint32).view(F32)[0]
    keep_prob = min(max(other / max(1.0 - top, 1e-9), 0.0), 1.0)
    fact = F32((1.0 - top) / max(other, 1e-9))
    g, h = g.copy(), np.ones_like(h)
    topm = np.abs(g) >= thresh
    seed = np.uint64(tree) * np.uint64(0x9E3779B97F4A7C15)
    with np.errstate(over="ignore"):
        hh = (gid.astype(np.uint64) ^ seed ^ GOSS_SALT) * np.uint64(0xD6E8FEB86659FD93)
    hh ^= hh >> np.uint64(32)
    keep = ((hh >> np.uint64(11)).astype(np.float64) / float(1 << 53)) < keep_prob
    other_m = ~topm & keep
    g[other_m] = g[other_m] * fact
    h[other_m] = fact
    return topm | other_m, g, h


def train_shard(bins, y, cuts, base, *, row_offset, n_global, n_trees, depth, n_bins,
                learning_rate=0.1, lambda_=1.0, min_child_h=1e-3, objective="l2",
                subsample=1.0, goss_top=0.0, goss_other=0.1, subtract=True, ex=None,
                expf=None):
    """Trains on this rank's rows (bins: [n_local, nf] u8) and returns the model dict,
    identical on every rank."""
    ex = ex or Exchange()
    n, nf = bins.shape
    nb1 = n_bins - 1
    leaves = 1 << depth
    lam, lr, mc = float(F32(lambda_)), float(F32(learning_rate)), float(F32(min_child_h))
    gid = np.arange(row_offset, row_offset + n, dtype=np.int64)
    pred = np.full(n, F32(base), F32)
    feat = np.zeros(n_trees * depth, np.uint32)
    thr = np.zeros(n_trees * depth, F32)
    thr_bin = np.zeros(n_trees * depth, np.uint32)
    leafval = np.zeros(n_trees * leaves, F32)
    fi_gain = np.zeros(nf, F32)
    fi_count = np.zeros(nf, F32)
    stride = 1
    if F32(subsample) < F32(0.999):
        stride = max(int(np.floor(1.0 / float(F32(subsample)) + 0.5)), 1)
    for t in range(n_trees):
        if objective == "logistic":
            e = np.array([expf(float(-v)) for v in pred], F32)
            pr = (F32(1.0) / (F32(1.0) + e)).astype(F32)
            g = (pr - y).astype(F32)
            h = np.maximum((pr * (F32(1.0) - pr)).astype(F32), F32(1e-6))
        else:
            g = (pred - y).astype(F32)
            h = np.ones(n, F32)
        if goss_top > 0:
            samp, g, h = goss_select(g, h, gid, n_global, float(F32(goss_top)),
                                     float(F32(goss_other)), t, ex)
        elif stride > 1:
            samp = gid % stride == t % stride
        else:
            samp = np.ones(n, bool)
        mx = np.array([f32_bits(np.abs(g[samp])).max(initial=0),
                       f32_bits(h[samp]).max(initial=0)], np.int64)
        mx = ex.max(mx)
        eg, eh = qscale_exp(int(mx[0])), qscale_exp(int(mx[1]))
        qg = np.where(samp, quantize(g, eg), 0)
        qh = np.where(samp, quantize(h, eh), 0)
        inv_g, inv_h = 2.0 ** -eg, 2.0 ** -eh
        wg, wh = wscale_exp(int(mx[0]), n_global), wscale_exp(int(mx[1]), n_global)
        node = np.zeros(n, np.int64)
        prev = None
        for level in range(depth):
            nn = 1 << level

            def build(groups, odd_only):
                hist = np.zeros((groups, nf, n_bins, 2), np.int64)
                rows = samp.copy()
                nd = node
                if odd_only:
                    rows &= (node & 1) == 1
                    nd = node >> 1
                r = np.nonzero(rows)[0]
                for f in range(nf):
                    np.add.at(hist[:, f, :, 0], (nd[r], bins[r, f]), qg[r])
                    np.add.at(hist[:, f, :, 1], (nd[r], bins[r, f]), qh[r])
                return ex.sum(hist.reshape(-1)).reshape(hist.shape)

            if level == 0 or not subtract:
                hist = build(nn, False)
            else:
                odd = build(nn // 2, True)
                hist = np.zeros((nn, nf, n_bins, 2), np.int64)
                hist[1::2] = odd
                hist[0::2] = prev - odd
            cs = np.cumsum(hist, axis=2)
            pg = cs[..., 0].astype(np.float64) * inv_g
            ph = cs[..., 1].astype(np.float64) * inv_h
            gain = np.zeros((nf, nb1))
            for nd in range(nn):
                gt, ht = pg[nd, :, nb1:], ph[nd, :, nb1:]
                parent = gt * gt / (ht + lam)
                gl, hl = pg[nd, :, :nb1], ph[nd, :, :nb1]
                gr, hr = gt - gl, ht - hl
                valid = ((hl >= mc) & (hr >= mc)).astype(np.float64)
                gain += valid * (gl * gl / (hl + lam) + gr * gr / (hr + lam) - parent)
            flat = int(np.argmax(gain.reshape(-1)))  # lowest (f, b) among the maxima
            bf, bb = flat // nb1, flat % nb1
            bg = float(gain[bf, bb])
            k = t * depth + level
            feat[k], thr[k], thr_bin[k] = bf, cuts[bf * nb1 + bb], bb
            fi_gain[bf] = F32(fi_gain[bf] + F32(max(bg, 0.0)))
            fi_count[bf] = F32(fi_count[bf] + F32(1.0))
            node = node * 2 + (bins[:, bf] > bb)
            prev = hist
        sg = np.zeros(leaves, np.int64)
        sh = np.zeros(leaves, np.int64)
        np.add.at(sg, node[samp], wquantize(g[samp], wg))
        np.add.at(sh, node[samp], wquantize(h[samp], wh))
        s = ex.sum(np.concatenate([sg, sh]))
        lg = s[:leaves].astype(np.float64) * 2.0 ** -wg
        lc = s[leaves:].astype(np.float64) * 2.0 ** -wh
        lv = (-lr * lg / (lc + lam)).astype(F32)
        leafval[t * leaves:(t + 1) * leaves] = lv
        pred = (pred + lv[node]).astype(F32)
    return dict(feat=feat, thr=thr, thr_bin=thr_bin, leafval=leafval, fi_gain=fi_gain,
                fi_count=fi_count)
