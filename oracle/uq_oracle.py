"""CPU restatement of UltraQuant's quantization hot path (test oracle).

TEST INFRASTRUCTURE ONLY -- never imported by the product package.

Every function cites the reference file:line it restates.  Floating-point
operations are written in the same order and precision as the reference so
that results agree bit-for-bit:

* numpy reductions along a contiguous last axis use numpy's pairwise sum
  (8 accumulators per block of <=128, halves split at a multiple of 8);
  the oracle calls numpy the same way, so the order is inherited.
* the Viterbi recurrence is evaluated with separate sub / square / add
  tensor ops (no fused multiply-add), min/argmin pick the first index.
* NEP-50 promotion: a float32 array times a numpy float64 scalar is float64.

Third-party arithmetic on the path (versions recorded in the golden
fixtures): numpy legacy ``RandomState`` (MT19937) for the sign vector and the
E8 calibration subsample, ``scipy.stats.norm.ppf`` for the codebook, torch
``min`` / ``argmin`` tie-breaking.
"""
from __future__ import annotations

import numpy as np
import torch

__all__ = [
    "next_pow2", "rht_signs", "rht_rows", "irht_rows", "d8_decode", "e8_decode",
    "entropy_bpw", "q_e8_fast", "E8_SCALE", "wnmse", "codebook", "pred_table",
    "trellis_quant", "trellis_quant_fast", "trellis_encode", "trellis_decode",
    "fwht_torch", "irht_torch", "recon_torch", "quant_trellis", "quant_step",
    "group_rms_f32", "viterbi_segments", "pack_states", "unpack_states", "enc_q8", "deq_q8",
    "hadamard28", "rht28_rows", "irht28_rows", "quant_step_b28", "q_uniform",
    "e8_codebook", "nearest_exact", "q_e8", "e8_bisect", "group_gn",
    "E8_SEARCH_FACTORS", "log2_table", "e8_scale_search_tables", "e8_scale_search_select", "e8_scale_search",
]


# ---------------------------------------------------------------------------
# Randomized Hadamard transform  (qlab.py:66-98)
# ---------------------------------------------------------------------------
def next_pow2(n: int) -> int:
    """qlab.py:66-69 -- smallest power of two >= n (1 for n <= 1)."""
    p = 1
    while p < n:
        p <<= 1
    return p


def rht_signs(n: int, seed: int = 0) -> np.ndarray:
    """qlab.py:78 and :96 -- legacy MT19937 ``choice([-1., 1.], n)``."""
    return np.random.RandomState(seed).choice([-1.0, 1.0], size=n)


def _butterflies(x: np.ndarray) -> np.ndarray:
    """Sylvester stages h = 1, 2, 4, ... n/2 along the last axis (qlab.py:80-84).

    For every pair (i, i+h) inside a block of 2h: new[i] = x[i] + x[i+h],
    new[i+h] = x[i] - x[i+h].  Stage order matters for rounding.
    """
    rows, n = x.shape
    h = 1
    while h < n:
        v = x.reshape(rows, n // (2 * h), 2, h)
        lo = v[:, :, 0, :]
        hi = v[:, :, 1, :]
        x = np.stack([lo + hi, lo - hi], axis=2).reshape(rows, n)
        h *= 2
    return x


def rht_rows(A: np.ndarray, seed: int = 0) -> np.ndarray:
    """qlab.py:71-85 -- pad columns to 2^k with zeros, multiply by the sign
    vector, run the butterflies in fp64, divide by sqrt(n)."""
    rows, n0 = A.shape
    n = next_pow2(n0)
    if n != n0:
        A = np.concatenate([A, np.zeros((rows, n - n0))], axis=1)
    d = rht_signs(n, seed)
    x = _butterflies(A * d)
    return x / np.sqrt(n)


def irht_rows(X: np.ndarray, n0: int, seed: int = 0) -> np.ndarray:
    """qlab.py:87-98 -- multiply by sqrt(n) (float32 input promotes to fp64),
    butterflies, then (x / n) * d and crop to n0 columns."""
    rows, n = X.shape
    x = X.copy() * np.sqrt(n)
    x = _butterflies(x)
    d = rht_signs(n, seed)
    x = (x / n) * d
    return x[:, :n0]


def wnmse(A: np.ndarray, Ah: np.ndarray) -> float:
    """qlab.py:53-54 -- sum((A - Ah)^2) / sum(A^2)."""
    return float(np.sum((A - Ah) ** 2) / np.sum(A ** 2))


# ---------------------------------------------------------------------------
# E8 nearest point  (qlab.py:133-183)
# ---------------------------------------------------------------------------
def d8_decode(Y: np.ndarray) -> np.ndarray:
    """qlab.py:133-142 -- nearest D8 point: round half to even; when the
    coordinate sum is odd, move the coordinate with the largest rounding error
    (first on ties) one step towards Y (np.sign, so an error of 0 moves 0)."""
    f = np.round(Y)
    parity = f.sum(1).astype(np.int64) % 2
    rows = np.nonzero(parity != 0)[0]
    if rows.size:
        err = Y[rows] - f[rows]
        k = np.argmax(np.abs(err), axis=1)
        f[rows, k] += np.sign(err[np.arange(rows.size), k])
    return f


def e8_decode(Y: np.ndarray) -> np.ndarray:
    """qlab.py:144-149 -- better of D8 and D8 + 1/2 (strict <, pairwise sums)."""
    a = d8_decode(Y)
    b = d8_decode(Y - 0.5) + 0.5
    da = ((Y - a) ** 2).sum(1)
    db = ((Y - b) ** 2).sum(1)
    return np.where((db < da)[:, None], b, a)


def entropy_bpw(idx_pts: np.ndarray) -> float:
    """qlab.py:151-156 -- empirical entropy of the 8-tuples 2*pts, / 8."""
    keys = np.ascontiguousarray((idx_pts * 2).astype(np.int64))
    keys = keys.view([("", np.int64)] * 8).ravel()
    _, cnt = np.unique(keys, return_counts=True)
    p = cnt / cnt.sum()
    return float(-(p * np.log2(p)).sum()) / 8.0


E8_SCALE: dict = {}


def e8_bisect(sub, target_bpw):
    """qlab.py:174-180 -- 18 halvings of [0.3, 10] on the entropy rate of the
    decoded sample `sub` (normalised 8-vectors in sample order)."""
    lo, hi = 0.3, 10.0
    for _ in range(18):
        mid = (lo + hi) / 2
        if entropy_bpw(e8_decode(sub / mid)) > target_bpw:
            lo = mid
        else:
            hi = mid
    return (lo + hi) / 2


def group_gn(A, group=256):
    """qlab.py:164-168 -- the normalised 8-vectors gn of A (fp64)."""
    flat = np.asarray(A).ravel().astype(np.float64)
    g = np.concatenate([flat, np.zeros((-flat.size) % group)]).reshape(-1, group)
    return (g / (np.sqrt((g ** 2).mean(1, keepdims=True)) + 1e-12)).reshape(-1, 8)


def q_e8_fast(A, target_bpw=2.0, group=256, calib_key="g", fixed_step=None,
              cache=None):
    """qlab.py:159-183 -- per-group RMS normalisation, one global step, E8.

    ``cache`` stands in for the module-global ``_E8_SCALE`` (qlab.py:158)."""
    cache = E8_SCALE if cache is None else cache
    flat = A.ravel().astype(np.float64)
    pad = (-flat.size) % group
    g = np.concatenate([flat, np.zeros(pad)]).reshape(-1, group)
    rms = np.sqrt((g ** 2).mean(1, keepdims=True)) + 1e-12
    gn = (g / rms).reshape(-1, 8)
    if fixed_step is not None:
        step = fixed_step
    else:
        if calib_key not in cache:
            ns = min(600_000, gn.shape[0])
            pick = np.random.RandomState(0).randint(0, gn.shape[0], ns)
            cache[calib_key] = e8_bisect(gn[pick], target_bpw)
        step = cache[calib_key]
    rec = (e8_decode(gn / step) * step).reshape(-1, group) * rms
    return rec.ravel()[:A.size].reshape(A.shape)


# ---------------------------------------------------------------------------
# Opt-in per-row scale search for the fixed-step E8 quantizer.  No counterpart
# in the reference (qlab.py:159-183 has one global step); this restatement
# DEFINES its parity.  For every row and each of 16 candidate steps
# step_c = step * 2^((c - 8) / 8) the row is decoded as q_e8_fast does it
# (per-256 group RMS, e8_decode(gn / step_c), rec = (p * step_c) * rms), and
#   D[r, c] = sum over the row of (A - rec)^2      (numpy order: per group,
#                                                   then over the row's groups)
#   H[r, c] = N log2 N - sum_v cnt_v log2 cnt_v     (bits of the row's N
#             lattice coordinates z = 2p under their own histogram; the sum
#             runs over z = -255 .. 255 in order, log2 from a table of the C
#             library's log2 of integers)
# Each row then takes c_r = first argmin_c D[r, c] + lam * H[r, c], with the
# smallest lam (bisection in exact midpoints) at which the total rate
# sum_r H[r, c_r] does not exceed that of the global step (c = 8): the same
# modelled rate, spent where it removes the most squared error.
# ---------------------------------------------------------------------------
E8_SEARCH_FACTORS = [float.fromhex(h) for h in (
    "0x1.0000000000000p-1", "0x1.172b83c7d517bp-1", "0x1.306fe0a31b715p-1", "0x1.4bfdad5362a27p-1",
    "0x1.6a09e667f3bcdp-1", "0x1.8ace5422aa0dbp-1", "0x1.ae89f995ad3adp-1", "0x1.d5818dcfba487p-1",
    "0x1.0000000000000p+0", "0x1.172b83c7d517bp+0", "0x1.306fe0a31b715p+0", "0x1.4bfdad5362a27p+0",
    "0x1.6a09e667f3bcdp+0", "0x1.8ace5422aa0dbp+0", "0x1.ae89f995ad3adp+0", "0x1.d5818dcfba487p+0")]
E8_SEARCH_BASE = 8            # the candidate equal to the given step
E8_SEARCH_ZMAX = 255          # |2p| bound of the rate histogram


def log2_table(n: int) -> np.ndarray:
    """log2(i) for i = 0 .. n from the C library (math.log2), 0 at i = 0."""
    import math
    return np.array([0.0] + [math.log2(i) for i in range(1, n + 1)], np.float64)


def e8_scale_search_tables(A, step, group=256):
    """(D, H) of shape (rows, 16) for the rotated matrix A (rows, n) fp64, n a
    multiple of `group`."""
    A = np.asarray(A, np.float64)
    rows, n = A.shape
    g = A.reshape(rows, n // group, group)
    rms = np.sqrt((g ** 2).mean(2, keepdims=True)) + 1e-12
    gn = g / rms
    LG = log2_table(n)
    D = np.empty((rows, 16))
    H = np.empty((rows, 16))
    for c, f in enumerate(E8_SEARCH_FACTORS):
        s = step * f
        p = e8_decode((gn / s).reshape(-1, 8)).reshape(g.shape)
        rec = (p * s) * rms
        D[:, c] = ((g - rec) ** 2).sum(axis=2).sum(axis=1)
        z = (p * 2).astype(np.int64).reshape(rows, n)
        if np.abs(z).max() > E8_SEARCH_ZMAX:
            raise ValueError("lattice coordinate beyond the rate histogram")
        for r in range(rows):
            cnt = np.bincount(z[r] + E8_SEARCH_ZMAX, minlength=2 * E8_SEARCH_ZMAX + 1)
            H[r, c] = n * LG[n] - np.cumsum(cnt * LG[cnt])[-1]
    return D, H


def e8_scale_search_select(D, H):
    """(choice per row, lam): the per-row candidates at the smallest lam whose
    total rate is at most the base step's (sequential sums over rows)."""
    def pick(lam):
        return np.argmin(D + lam * H, axis=1)

    def rate(c):
        return float(np.cumsum(H[np.arange(H.shape[0]), c])[-1])

    r0 = float(np.cumsum(H[:, E8_SEARCH_BASE])[-1])
    if rate(pick(0.0)) <= r0:
        return pick(0.0), 0.0
    hi = 1.0
    for _ in range(400):
        if rate(pick(hi)) <= r0:
            break
        hi *= 2.0
    lo = 0.0
    for _ in range(64):
        mid = (lo + hi) * 0.5
        if rate(pick(mid)) <= r0:
            hi = mid
        else:
            lo = mid
    return pick(hi), hi


def e8_scale_search(A, step, group=256):
    """Opt-in per-row scale search on the rotated matrix A: returns (rec fp64,
    choice per row, lam) with rec the q_e8_fast reconstruction at each row's
    chosen step."""
    A = np.asarray(A, np.float64)
    rows, n = A.shape
    D, H = e8_scale_search_tables(A, step, group)
    choice, lam = e8_scale_search_select(D, H)
    g = A.reshape(rows, n // group, group)
    rms = np.sqrt((g ** 2).mean(2, keepdims=True)) + 1e-12
    s = (step * np.array(E8_SEARCH_FACTORS))[choice][:, None, None]
    p = e8_decode(((g / rms) / s).reshape(-1, 8)).reshape(g.shape)
    rec = ((p * s) * rms).reshape(rows, n)
    return rec, choice, lam


# ---------------------------------------------------------------------------
# Bitshift trellis  (trellis.py:14-108, qat.py:11-59)
# ---------------------------------------------------------------------------
def codebook(L: int, seed: int = 0) -> np.ndarray:
    """trellis.py:14-19 -- 64-bit mix hash of the state, low 32 bits to
    u in (0, 1), inverse normal CDF, rounded to float32.  ``seed`` is unused
    by the reference and therefore here."""
    from scipy.stats import norm
    s = np.arange(1 << L, dtype=np.uint64)
    h = s * np.uint64(2654435761) + np.uint64(0x9E3779B97F4A7C15)
    h ^= h >> np.uint64(29)
    h *= np.uint64(0xBF58476D1CE4E5B9)
    h ^= h >> np.uint64(32)
    u = ((h & np.uint64(0xFFFFFFFF)).astype(np.float64) + 0.5) / 2 ** 32
    return norm.ppf(u).astype(np.float32)


def pred_table(L: int, R: int) -> np.ndarray:
    """trellis.py:21-25 -- pred[s, k] = ((s >> R) | (k << (L-R))) & (2^L - 1)."""
    S = 1 << L
    s = np.arange(S)[:, None]
    k = np.arange(1 << R)[None, :]
    return ((s >> R) | (k << (L - R))) & (S - 1)


def group_rms_f32(g: np.ndarray) -> np.ndarray:
    """trellis.py:75 -- float32 sqrt(mean(g^2)) + 1e-12 along the last axis."""
    return np.sqrt((g ** 2).mean(-1, keepdims=True)) + 1e-12


def viterbi_segments(xn: np.ndarray, L: int, R: int, cw=None, chunk: int = 1 << 16):
    """trellis.py:84-105 (= qat.py:141-152) -- min-plus Viterbi per row of
    ``xn`` (nseq, T) float32.  Returns the int64 state path (nseq, T).

    Forward: cost_0[s] = (x_0 - cw[s])^2; for t >= 1
    m[q] = min_k cost[k*2^(L-R) + q] (first k on ties), bp[t, q] = k,
    cost[s] = (x_t - cw[s])^2 + m[s >> R].  Backward from the first argmin:
    s_{t-1} = bp[t, s_t >> R] * 2^(L-R) + (s_t >> R).
    """
    cw_t = torch.from_numpy(codebook(L) if cw is None else np.asarray(cw, np.float32))
    nseq, T = xn.shape
    Q = 1 << (L - R)
    K = 1 << R
    out = np.empty((nseq, T), np.int64)
    cw2 = cw_t[None, :]
    for c0 in range(0, nseq, chunk):
        x = torch.from_numpy(np.ascontiguousarray(xn[c0:c0 + chunk], np.float32))
        b = x.shape[0]
        cost = (x[:, 0:1] - cw2) ** 2
        bp = torch.empty((b, T, Q), dtype=torch.uint8)
        for t in range(1, T):
            m, k = cost.view(b, K, Q).min(dim=1)
            bp[:, t, :] = k.to(torch.uint8)
            cost = (x[:, t:t + 1] - cw2) ** 2 + m.repeat_interleave(K, dim=1)
        st = torch.empty((b, T), dtype=torch.long)
        st[:, T - 1] = cost.argmin(1)
        rows = torch.arange(b)
        for t in range(T - 1, 0, -1):
            q = st[:, t] >> R
            st[:, t - 1] = bp[rows, t, q].long() * Q + q
        out[c0:c0 + b] = st.numpy()
    return out


def _flat_normalise(A, seg, scale_group):
    """trellis.py:69-80 -- float32 flatten, zero-pad to the scale group,
    per-group RMS, normalise, cut into Viterbi segments."""
    flat = A.astype(np.float32).ravel()
    pad = (-flat.size) % scale_group
    g = np.concatenate([flat, np.zeros(pad, np.float32)]).reshape(-1, scale_group)
    sc_g = group_rms_f32(g)
    xn = (g / sc_g).ravel().reshape(-1, seg)
    return xn, sc_g, flat.size, pad


def trellis_quant_fast(A, L=12, R=2, seg=64, scale_group=256, mem_gb=3.0):
    """trellis.py:62-108 -- segmented Viterbi; returns cw[s] * sc_g (float32).
    ``mem_gb`` bounds the backpointer chunk as in trellis.py:81 (numerically
    irrelevant)."""
    nrow, ncol = A.shape
    cw = codebook(L)
    xn, sc_g, ntot, _ = _flat_normalise(A, seg, scale_group)
    chunk = max(1, int(mem_gb * 1e9 / (seg * (1 << L))))
    st = viterbi_segments(xn, L, R, cw, chunk=chunk)
    rec = cw[st].ravel()
    rec = (rec.reshape(-1, scale_group) * sc_g).ravel()
    return rec[:ntot].reshape(nrow, ncol).astype(np.float32)


def trellis_encode(A, L=12, R=2, seg=64, scale_group=256):
    """qat.py:11-33 -- same Viterbi; returns (states int32, sc_g, cw, meta)."""
    nrow, ncol = A.shape
    cw = codebook(L)
    xn, sc_g, ntot, pad = _flat_normalise(A, seg, scale_group)
    st = viterbi_segments(xn, L, R, cw).astype(np.int32)
    meta = dict(nrow=nrow, ncol=ncol, Ntot=ntot, seg=seg, scale_group=scale_group,
                pad=pad, Nseg=st.shape[0])
    return st, sc_g.astype(np.float32), cw, meta


def trellis_decode(states, cw, sc_g, meta):
    """trellis.py:104-108 -- cw[states] * sc_g, cropped to Ntot (float32)."""
    rec = np.asarray(cw, np.float32)[states].ravel()
    rec = (rec.reshape(-1, meta["scale_group"]) * sc_g).ravel()
    return rec[:meta["Ntot"]].reshape(meta["nrow"], meta["ncol"]).astype(np.float32)


def trellis_quant(A, L=10, R=2, group=256, chunk_rows=512):
    """trellis.py:27-60 -- full-row Viterbi (one sequence per padded row) with
    per-(row, group) RMS; returns float32 reconstruction."""
    del chunk_rows
    cw = codebook(L)
    nrow, T = A.shape
    out = np.empty((nrow, T), np.float32)
    blk = A.astype(np.float32)
    Tp = ((T + group - 1) // group) * group
    pad = np.zeros((nrow, Tp), np.float32)
    pad[:, :T] = blk
    g = pad.reshape(nrow, Tp // group, group)
    sc = group_rms_f32(g)
    xn = (g / sc).reshape(nrow, Tp)
    st = viterbi_segments(xn, L, R, cw)
    rec = (cw[st].reshape(nrow, Tp // group, group) * sc).reshape(nrow, Tp)
    out[:] = rec[:, :T]
    return out


def fwht_torch(x):
    """qat.py:35-41 -- differentiable FWHT along the last axis, / sqrt(n)."""
    n = x.shape[-1]
    shape = x.shape
    h = 1
    while h < n:
        v = x.reshape(-1, n // (2 * h), 2, h)
        x = torch.cat([v[:, :, 0, :] + v[:, :, 1, :], v[:, :, 0, :] - v[:, :, 1, :]],
                      dim=2).reshape(*shape[:-1], n)
        h *= 2
    return x / np.sqrt(n)


def irht_torch(Xrot, in0, seed=0):
    """qat.py:43-49 -- fwht_torch(X) * d, cropped to in0."""
    n = Xrot.shape[1]
    x = fwht_torch(Xrot)
    d = torch.tensor(rht_signs(n, seed), dtype=Xrot.dtype, device=Xrot.device)
    return (x * d)[:, :in0]


def recon_torch(states, cw, sc_g, meta, sH, in0):
    """qat.py:51-59 -- cw[states] * sc_g -> irht_torch -> / sH."""
    dev = cw.device
    st = torch.as_tensor(states, device=dev, dtype=torch.long)
    rec = cw[st].reshape(-1)[:meta["Nseg"] * meta["seg"]]
    rec = (rec.reshape(-1, meta["scale_group"]) * sc_g).reshape(-1)[:meta["Ntot"]]
    return irht_torch(rec.reshape(meta["nrow"], meta["ncol"]), in0) / sH


# ---------------------------------------------------------------------------
# Builder recipes around the path  (buildtrellis.py:16-20, buildalloc.py:21-24)
# ---------------------------------------------------------------------------
def quant_trellis(W, H, L=12, R=2, seg=64, scale_group=256):
    """buildtrellis.py:16-20 -- clamp H, A = W*sqrt(H), RHT, trellis, iRHT, /sqrt(H)."""
    H = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(H)[None, :]
    A = W * sH
    in0 = A.shape[1]
    Ah = irht_rows(trellis_quant_fast(rht_rows(A), L=L, R=R, seg=seg,
                                      scale_group=scale_group), in0)
    return (Ah / sH).astype(np.float32)


def quant_step(W, H, step):
    """buildalloc.py:21-24 -- same recipe with E8 at a fixed step."""
    H = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(H)[None, :]
    Ah = irht_rows(q_e8_fast(rht_rows(W * sH), fixed_step=step), W.shape[1])
    return (Ah / sH).astype(np.float32)


# ---------------------------------------------------------------------------
# Packed state paths (qat.py:11-33 states; the L + R (T-1) bits per sequence
# behind the reference's bits-per-weight accounting)
# ---------------------------------------------------------------------------
def pack_states(states, L, R):
    """S = s_0 2^(R(T-1)) + sum_t (s_t mod 2^R) 2^(R(T-1-t)) per sequence, as
    little-endian 32-bit words (Python integers; small cases only)."""
    st = np.asarray(states, dtype=np.int64)
    nseq, T = st.shape
    words = (L + R * (T - 1) + 31) // 32
    out = np.zeros((nseq, words), dtype=np.uint32)
    for i in range(nseq):
        S = int(st[i, 0]) & ((1 << L) - 1)
        for t in range(1, T):
            S = (S << R) | (int(st[i, t]) & ((1 << R) - 1))
        for w in range(words):
            out[i, w] = (S >> (32 * w)) & 0xFFFFFFFF
    return out


def unpack_states(packed, T, L, R):
    """Inverse of pack_states: s_t = (S >> R(T-1-t)) mod 2^L."""
    pk = np.asarray(packed, dtype=np.uint32)
    out = np.zeros((pk.shape[0], T), dtype=np.int32)
    for i in range(pk.shape[0]):
        S = 0
        for w in range(pk.shape[1]):
            S |= int(pk[i, w]) << (32 * w)
        for t in range(T):
            out[i, t] = (S >> (R * (T - 1 - t))) & ((1 << L) - 1)
    return out


# ---------------------------------------------------------------------------
# Q8_0 blocks (buildq.py:21-30 enc_q8, qlab.py:27-32 deq_q8)
# ---------------------------------------------------------------------------
def enc_q8(W):
    """buildq.py:21-30: per 32-block float16(max|x|/127) + int8 round-half-even."""
    rows, cols = W.shape
    nb = cols // 32
    x = W.reshape(rows, nb, 32).astype(np.float32)
    sc = np.max(np.abs(x), 2, keepdims=True) / 127.0
    sc = np.where(sc == 0, 1e-9, sc)
    q = np.round(x / sc).clip(-127, 127).astype(np.int8)
    out = np.zeros((rows, nb, 34), np.uint8)
    out[:, :, :2] = sc.squeeze(-1).astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, nb * 34)


def deq_q8(data):
    """qlab.py:27-32 on the raw (rows, nb*34) block bytes."""
    rows, brow = data.shape
    nb = brow // 34
    d = data.reshape(rows, nb, 34)
    sc = d[:, :, :2].copy().view(np.float16).astype(np.float32)
    qs = d[:, :, 2:].view(np.int8).astype(np.float32)
    return (sc * qs).reshape(rows, nb * 32)


# ---------------------------------------------------------------------------
# Opt-in block-factorised RHT for n0 = 28 * 2^m (no counterpart in the
# reference, which pads to a power of two; parity of this mode is defined by
# this restatement alone).  H_28 is the Paley type-I Hadamard matrix over
# GF(27) = GF(3)[x] / (x^3 - x - 1); the transform is (H_28 (x) H_P) D / sqrt(N)
# with the normalisation applied as a multiplication by RN(1 / sqrt(N)).
# ---------------------------------------------------------------------------
def hadamard28() -> np.ndarray:
    """28 x 28 +-1 matrix with H H^T = 28 I (Paley construction, q = 27)."""
    import itertools

    def mul(a, b):
        r = [0] * 5
        for i in range(3):
            for j in range(3):
                r[i + j] = (r[i + j] + a[i] * b[j]) % 3
        for k in (4, 3):                      # x^3 = x + 1
            c, r[k] = r[k], 0
            r[k - 3] = (r[k - 3] + c) % 3
            r[k - 2] = (r[k - 2] + c) % 3
        return tuple(r[:3])

    elems = list(itertools.product(range(3), repeat=3))
    zero = (0, 0, 0)
    squares = {mul(a, a) for a in elems if a != zero}

    def chi(a):
        return 0 if a == zero else (1 if a in squares else -1)

    Q = np.array([[chi(tuple((x - y) % 3 for x, y in zip(a, b))) for b in elems] for a in elems])
    H = np.zeros((28, 28), dtype=np.int64)
    H[0, :] = 1
    H[1:, 0] = -1
    H[1:, 1:] = Q + np.eye(27, dtype=np.int64)
    return H


def _fwht_blocks(x, P):
    """Sylvester butterflies h = 1 .. P/2 inside each P-block of the rows."""
    rows, N = x.shape
    x = x.reshape(rows, N // P, P)
    h = 1
    while h < P:
        v = x.reshape(rows, N // P, P // (2 * h), 2, h)
        a, b = v[:, :, :, 0, :], v[:, :, :, 1, :]
        x = np.concatenate([a + b, a - b], axis=3).reshape(rows, N // P, P)
        h *= 2
    return x.reshape(rows, N)


def _mix28(x, P, transpose):
    """z[i] = sum_k H[i, k] y[k] (or H^T) over the 28 blocks, accumulated
    k = 0 .. 27 in order from +-y[0]."""
    H = hadamard28()
    M = H.T if transpose else H
    rows, N = x.shape
    y = x.reshape(rows, 28, P)
    z = np.empty_like(y)
    for i in range(28):
        acc = y[:, 0, :] if M[i, 0] > 0 else -y[:, 0, :]
        for k in range(1, 28):
            acc = acc + y[:, k, :] if M[i, k] > 0 else acc - y[:, k, :]
        z[:, i, :] = acc
    return z.reshape(rows, N)


def rht28_rows(A, seed=0):
    """Opt-in forward transform for n0 = 28 P (P a power of two >= 16)."""
    A = np.asarray(A, dtype=np.float64)
    rows, N = A.shape
    P = N // 28
    assert N == 28 * P and P >= 16 and P & (P - 1) == 0
    d = rht_signs(N, seed)
    x = _fwht_blocks(A * d, P)
    x = _mix28(x, P, transpose=False)
    return x * (1.0 / np.sqrt(float(N)))


def irht28_rows(X, seed=0):
    """Inverse of rht28_rows: H^T mix, block butterflies, * RN(1/sqrt(N)), * d."""
    X = np.asarray(X, dtype=np.float64)
    rows, N = X.shape
    P = N // 28
    x = _mix28(X, P, transpose=True)
    x = _fwht_blocks(x, P)
    return (x * (1.0 / np.sqrt(float(N)))) * rht_signs(N, seed)


def quant_step_b28(W, H, step):
    """Opt-in buildalloc recipe with the block-factorised transform:
    What = irht28(q_e8_fast(rht28(W sH), fixed_step)) / sH (float32)."""
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    X = rht28_rows(np.asarray(W, np.float64) * sH)
    Xq = q_e8_fast(X, fixed_step=step)
    return (irht28_rows(Xq) / sH).astype(np.float32), X, Xq


def q_uniform(A, bpw, bs=32):
    """qlab.py:100-106: per-block absmax, rint(x / amax * lvl) / lvl * amax."""
    x = A.reshape(-1, bs)
    amax = np.max(np.abs(x), axis=1, keepdims=True) + 1e-12
    lvl = (1 << (int(round(bpw)) - 1)) - 1
    return (np.round(x / amax * lvl) / lvl * amax).reshape(A.shape)


# ---------------------------------------------------------------------------
# Finite-codebook E8 quantizer  (qlab.py:110-124, 185-198)
# ---------------------------------------------------------------------------
_E8CB: dict = {}
_E8PTS: list = []


def _e8_points():
    """(D8 grid points as int8, norms of the point list, argsort of the norms)."""
    if not _E8PTS:
        g = (np.indices((7,) * 8, dtype=np.int8).reshape(8, -1).T - 3).astype(np.int8)
        d8 = g[(g.astype(np.int64).sum(1) % 2) == 0]
        n_d8 = (d8.astype(np.int64) ** 2).sum(1)
        n_half = ((2 * d8.astype(np.int64) + 1) ** 2).sum(1) // 4    # |p + 1/2|^2, an integer
        norms = np.concatenate([n_d8, n_half]).astype(np.float64)
        _E8PTS.extend([d8, norms, np.argsort(norms)])
    return _E8PTS


def e8_codebook(K):
    """qlab.py:111-124: the points of D8 (even coordinate sum, coordinates in
    [-3, 3]) followed by the same points plus 1/2, both in grid order (first
    coordinate slowest); the K of smallest norm by np.argsort (numpy's order
    among equal norms), divided by sqrt(mean |p|^2 / 8)."""
    if K not in _E8CB:
        d8, _, order = _e8_points()
        ids = order[:K]
        pts = d8[ids % len(d8)].astype(np.float64) + np.where(ids >= len(d8), 0.5, 0.0)[:, None]
        _E8CB[K] = pts / np.sqrt((pts ** 2).sum(1).mean() / 8)
    return _E8CB[K]


def nearest_exact(X, cb, chunk=2048):
    """Exact Euclidean nearest neighbour (what cKDTree.query returns for
    eps = 0): fp64 distances sum_i (x_i - c_i)^2 in coordinate order, the
    smallest, lowest index on equal distances."""
    out = np.empty(len(X), np.int64)
    for s in range(0, len(X), chunk):
        x = X[s:s + chunk]
        d = np.zeros((len(x), len(cb)))
        for i in range(X.shape[1]):
            e = x[:, i:i + 1] - cb[None, :, i]
            d = d + e * e
        out[s:s + chunk] = np.argmin(d, axis=1)
    return out


def q_e8(A, bpw, group_scale=256):
    """qlab.py:185-198: zero-pad the flattened A (fp64) to whole groups,
    s = sqrt(mean(g^2)) + 1e-12 per group, gn = g / s as 8-vectors, out =
    cb[nearest] * s."""
    K = 1 << int(round(bpw * 8))
    cb = e8_codebook(K)
    flat = np.asarray(A).ravel().astype(np.float64)
    flat = np.concatenate([flat, np.zeros((-flat.size) % group_scale)])
    g = flat.reshape(-1, group_scale)
    s = np.sqrt((g ** 2).mean(1, keepdims=True)) + 1e-12
    gn = (g / s).reshape(-1, 8)
    if not np.isfinite(gn).all():
        raise ValueError("'x' must be finite, check for nan or inf values")
    idx = nearest_exact(gn, cb)
    rec = (cb[idx].reshape(-1, group_scale) * s).ravel()[:np.asarray(A).size]
    return rec.reshape(np.shape(A))
