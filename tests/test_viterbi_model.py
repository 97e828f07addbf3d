"""CPU model of the Viterbi kernel's work decomposition, checked against the oracle.

The model follows ``ultraquant_b200/csrc/uq_trellis.cu`` index by index:
thread v owns q in [NQ*v, NQ*v + NQ) (64 states), reads
m_{t-1}[k*Rn + r] for its r-range and writes one decision record per step,
which the traceback decodes:

* R = 1, 4: the tournament's first-index argmin from sign bits of candidate
  differences, R-bit field of q-local jq at bits [jq*R, jq*R + R) of one
  32-bit word;
* R = 2, 3: m = min_k c_k and the raw signs s_k = signbit(m - c_k), k < K-1
  (the first clear one is the first-index argmin), in two 32-bit words: word
  jq // HQ, pair pw = (jq % HQ) // 2 at bits 2F*pw .. 2F*pw + 2F, s_k at bit
  2F*pw + 2k + (jq & 1), F = K - 1, HQ = NQ / 2.

It also checks that the shared-memory swizzles are bijections and
bank-conflict free for the access patterns of every (L, R) the kernel is
built for.
"""
import numpy as np
import pytest

import oracle as O

SWZ = {1: (3, 7), 2: (2, 7), 3: (1, 7), 4: (1, 0)}


def _sign(x):
    return np.signbit(np.float32(x))


def _tourney(c):
    """min and first-index argmin of candidates c (float32) via the kernel's
    level-by-level min + sign-of-difference selection."""
    K = len(c)
    R = K.bit_length() - 1
    val = list(np.float32(v) for v in c)
    P = [[None] * K for _ in range(R)]
    for lev in range(1, R + 1):
        for i in range(K >> lev):
            d = np.float32(val[2 * i + 1] - val[2 * i])
            s = _sign(d)
            for j in range(lev - 1):
                P[j][i] = P[j][2 * i + 1] if s else P[j][2 * i]
            P[lev - 1][i] = s
            val[i] = np.float32(min(val[2 * i], val[2 * i + 1]))
    k = sum(int(P[j][0]) << j for j in range(R))
    return val[0], k


def record_layout(R):
    """(raw, F, words per record, q per word) of the kernel's decision record."""
    K = 1 << R
    NQ = 64 // K
    raw = R in (2, 3)
    F = K - 1 if raw else R
    bpw = (NQ * F + 31) // 32
    return raw, F, bpw, NQ // bpw


def _gpu_signbit(d):
    """Sign bit of a float32 difference as the GPU produces it: inf - inf is
    the canonical NaN 0x7FFFFFFF (sign clear), not x86's 0xFFC00000."""
    return False if np.isnan(d) else bool(np.signbit(d))


def _raw_signs(c):
    """min of the candidates and s_k = signbit(m - c_k) for k < K - 1."""
    m = np.float32(min(c))
    with np.errstate(invalid="ignore"):
        return m, [_gpu_signbit(np.float32(m - ck)) for ck in c[:-1]]


def model_viterbi(x, L, R, cw):
    """One sequence x (T,) float32 through the kernel's decomposition."""
    K = 1 << R
    Q = 1 << (L - R)
    Rn = Q >> R
    NQ = 64 // K
    TPS = Q // NQ
    NR = NQ // K if NQ >= K else 1
    T = len(x)
    raw, F, bpw, HQ = record_layout(R)
    m_prev = None
    words = np.zeros((max(T - 1, 0), TPS, bpw), np.uint64)
    for t in range(T - 1):
        m_new = np.empty(Q, np.float32)
        for v in range(TPS):
            r0 = (NQ * v) >> R
            mloc = None
            if m_prev is not None:
                mloc = [[m_prev[k * Rn + r0 + i] for i in range(NR)] for k in range(K)]
            rec = [0] * bpw
            for jq in range(NQ - 1, -1, -1):
                i = (jq >> R) if NQ >= K else 0
                q = NQ * v + jq
                c = []
                for k in range(K):
                    d = np.float32(x[t] - cw[k * Q + q])
                    d = np.float32(d * d)
                    if mloc is not None:
                        d = np.float32(d + mloc[k][i])
                    c.append(d)
                w = jq // HQ
                if raw:
                    mn, s = _raw_signs(c)
                    base = 2 * F * ((jq % HQ) // 2) + (jq & 1)
                    for k in range(F):
                        rec[w] |= int(s[k]) << (base + 2 * k)
                else:
                    mn, kk = _tourney(c)
                    rec[w] |= kk << (F * (jq % HQ))
                m_new[q] = mn
            for w in range(bpw):
                assert rec[w] < (1 << 32)
                words[t, v, w] = rec[w]
        m_prev = m_new
    # final argmin over all states (first index)
    best_v, best_s = None, None
    S = 1 << L
    for s in range(S):
        d = np.float32(x[T - 1] - cw[s])
        d = np.float32(d * d)
        if m_prev is not None:
            d = np.float32(d + m_prev[s >> R])
        if best_v is None or d < best_v:
            best_v, best_s = d, s
    # traceback
    st = np.empty(T, np.int64)
    s = best_s
    st[T - 1] = s
    for t in range(T - 1, 0, -1):
        q = s >> R
        jq = q % NQ
        w = int(words[t - 1, q // NQ, jq // HQ])
        if raw:
            bits = w >> (2 * F * ((jq % HQ) // 2) + (jq & 1))
            k = next((j for j in range(F) if not (bits >> (2 * j)) & 1), F)
        else:
            k = (w >> (F * (jq % HQ))) & ((1 << F) - 1)
        s = k * Q + q
        st[t - 1] = s
    return st


@pytest.mark.parametrize("L,R", [(6, 1), (6, 2), (6, 3), (8, 4), (7, 2), (8, 3), (9, 2), (10, 3)])
def test_model_matches_oracle(L, R):
    rng = np.random.RandomState(L * 10 + R)
    cw = O.codebook(L)
    for T in (1, 2, 9):
        x = rng.randn(3, T).astype(np.float32)
        x[0, :] = np.round(x[0, :])          # exact values provoke cost ties
        ref = O.viterbi_segments(x, L, R, cw)
        for b in range(3):
            assert np.array_equal(model_viterbi(x[b], L, R, cw), ref[b])


def test_tourney_first_index():
    rng = np.random.RandomState(0)
    for K in (2, 4, 8, 16):
        for _ in range(300):
            c = np.round(rng.rand(K) * 3).astype(np.float32)  # many ties
            mn, k = _tourney(c)
            assert mn == c.min() and k == int(np.argmin(c))


def test_raw_signs_first_index():
    """The lowest clear s_k = signbit(m - c_k) is torch's first-index argmin,
    on ties, zeros, infinities and values a few ulps apart."""
    rng = np.random.RandomState(1)
    specials = np.array([0.0, np.inf, 1.0, np.nextafter(np.float32(1), np.float32(2)), 3e-39, 1e-45],
                        np.float32)
    for K in (4, 8):
        for it in range(2000):
            if it % 2:
                c = np.round(rng.rand(K) * 3).astype(np.float32)
            else:
                c = rng.choice(specials, K).astype(np.float32)
            mn, s = _raw_signs(list(c))
            k = next((j for j, b in enumerate(s) if not b), K - 1)
            assert mn == c.min() and k == int(np.argmin(c))


@pytest.mark.parametrize("R", [1, 2, 3, 4])
def test_record_fits(R):
    raw, F, bpw, HQ = record_layout(R)
    NQ = 64 // (1 << R)
    assert bpw in (1, 2) and HQ * bpw == NQ and HQ * F <= 32
    assert raw == (R in (2, 3))


def _conflict_ways_128(chunks):
    worst = 1
    for q in range(4):
        cs = set(c for c in chunks[q * 8:(q + 1) * 8])
        groups = {}
        for c in cs:
            groups.setdefault(c % 8, set()).add(c)
        worst = max([worst] + [len(g) for g in groups.values()])
    return worst


@pytest.mark.parametrize("R", [1, 2, 3, 4])
def test_swizzle_bijective_and_conflict_free(R):
    a, m = SWZ[R]
    K = 1 << R
    NQ = 64 // K
    for L in range(max(6, 2 * R), 17):
        Q = 1 << (L - R)
        QC = Q // 4
        P = lambda c: c ^ ((c >> a) & m)  # noqa: E731
        nch = min(QC * max(1, 512 // max(Q // NQ, 1)), 1 << 16)
        assert sorted(P(c) for c in range(nch)) == list(range(nch))
        if L < 11:
            continue  # small tables: a few 2-way conflicts are accepted
        TPS = Q // NQ
        for w0 in range(0, min(TPS, 512), 32):
            lanes = range(w0, w0 + 32)
            for c in range(NQ // 4):
                assert _conflict_ways_128([P(NQ * v // 4 + c) for v in lanes]) == 1
            G = NQ // K
            if G >= 4:
                Rn = Q // K
                for k in range(K):
                    for i4 in range(G // 4):
                        assert _conflict_ways_128([P((k * Rn + G * v) // 4 + i4) for v in lanes]) == 1
