"""CPU model of the shared-memory accesses of ``rht_tma_kernel`` and
``rht_halves_kernel`` (ultraquant_b200/csrc/uq_rht.cu), index by index, and
of the halves kernel's data flow.

For every warp instruction that touches shared memory -- pass 0's 16-byte
loads from the 128-byte-swizzled lines, the stores and loads of each
transpose through the element-swizzled tile (swz(E) = E ^ ((E >> 4) & 15)),
the inbox writes and reads of rows of 32768, and the epilogue's stores into
the swizzled output lines -- the model lists the 32 lanes' byte addresses and
counts the wavefronts a bank-conflict-free access needs (bytes / 128) against
the most distinct 4-byte words any one of the 32 banks receives.  Equal
counts mean no bank conflict.  The layouts are also checked to be
permutations (every element written once, read back from where it was put).

One access is not conflict-free, and is pinned as such: with rows of 8192
columns (LB = 13) and float32 output, the epilogue's half-warps write 16
consecutive floats each into lines 4096 elements apart, which the 128-byte
swizzle maps onto the same 16 banks (2 wavefronts for 128 bytes).  Only the
trellis pipeline's forward transform of rows of 8192 writes float32 this
way, a small share of its step; fp64 outputs (rht_rows, E8) are
conflict-free, and the halves kernel stores from registers.
"""
import pytest

BANKS = 32


def swz(e):
    return e ^ ((e >> 4) & 15)


def swz128(e, size):
    epl, epc = 128 // size, 16 // size
    r, c = e // epl, (e % epl) // epc
    return r * 128 + ((c ^ (r & 7)) << 4) + (e % epc) * size


def wavefronts(addrs, width):
    """(needed, ideal) wavefronts of one warp access of `width` bytes per lane."""
    words = {}
    for a in addrs:
        for w in range(a // 4, (a + width) // 4):
            words.setdefault(w % BANKS, set()).add(w)
    need = max(len(v) for v in words.values())
    ideal = max(1, (len(set(addrs)) * width + 127) // 128)
    return need, ideal


def elem12(tid, j):
    return (tid & 15) | (((tid >> 5) & 15) << 4) | (j << 8) | (((tid >> 4) & 1) << 12)


def out_idx(tid, j, LB):
    """Column of register j's output in rht_tma_kernel (rows of 2^LB)."""
    if LB == 13:
        return elem12(tid, j)
    return tid + (j << (LB - 4))


def pass_accesses(LB, in_size, lanes):
    """Pass 0's loads from the swizzled lines and the transposes' stores and
    loads through the element-swizzled tile, for one warp and one 2^LB part."""
    shfl12 = LB == 13
    if in_size == 8:
        for c in range(8):
            yield "pass0", 16, [t * 128 + ((c ^ (t & 7)) << 4) for t in lanes]
    else:
        for c in range(4):
            yield "pass0", 16, [(t >> 1) * 128 + (((4 * (t & 1) + c) ^ ((t >> 1) & 7)) << 4) for t in lanes]
    # transposes: bits [p, p + 4) after bits [prev, prev + 4)
    prev = 0
    p = 4
    while p - 4 < (8 if shfl12 else LB - 4):
        pp = min(p, LB - 4)
        for j in range(16):
            yield f"T{pp}.st", 8, [8 * swz((t & ((1 << prev) - 1)) | ((t >> prev) << (prev + 4)) + (j << prev))
                                   for t in lanes]
        for j in range(16):
            if shfl12 and pp == 8:
                yield f"T{pp}.ld", 8, [8 * swz(elem12(t, 0) + (j << pp)) for t in lanes]
            else:
                yield f"T{pp}.ld", 8, [8 * swz((t & ((1 << pp) - 1)) | ((t >> pp) << (pp + 4)) + (j << pp))
                                       for t in lanes]
        prev = pp
        p += 4


def kernel_accesses(LB, in_size, out_size):
    """rht_tma_kernel: (name, width, [32 addresses]) for every warp access of one row."""
    NT = 1 << (LB - 4)
    for w in range(NT // 32):
        lanes = range(32 * w, 32 * w + 32)
        yield from pass_accesses(LB, in_size, lanes)
        # epilogue stores into the swizzled output lines
        for j in range(16):
            yield "epilogue.st", out_size, [swz128(out_idx(t, j, LB), out_size) for t in lanes]


def halves_accesses(in_size, CL):
    """rht_halves_kernel: both 8192-element parts of a CTA take the passes of
    the rows of 8192; rows of 32768 (CL = 2) add the inbox's 8-byte writes
    (st.async from the partner) and reads at 8 elem12(j).  Its results go to
    global memory straight from registers."""
    for w in range(512 // 32):
        lanes = range(32 * w, 32 * w + 32)
        for _ in range(2):
            yield from pass_accesses(13, in_size, lanes)
        if CL == 2:
            for j in range(16):
                yield "inbox.st", 8, [8 * elem12(t, j) for t in lanes]
                yield "inbox.ld", 8, [8 * elem12(t, j) for t in lanes]


CASES = [(12, 8, 8), (12, 4, 4), (12, 4, 8), (12, 8, 4), (13, 8, 8), (13, 4, 4), (13, 4, 8), (13, 8, 4)]


@pytest.mark.parametrize("LB,isz,osz", CASES)
def test_rht_tma_shared_accesses_conflict_free(LB, isz, osz):
    for name, width, addrs in kernel_accesses(LB, isz, osz):
        need, ideal = wavefronts(addrs, width)
        if name == "epilogue.st" and LB == 13 and osz == 4:
            assert (need, ideal) == (2, 1), f"{name}: {need} wavefronts (known 2-way case)"
            continue
        assert need == ideal, f"{name}: {need} wavefronts, {ideal} without conflicts"


@pytest.mark.parametrize("isz,CL", [(8, 1), (4, 1), (8, 2), (4, 2)])
def test_rht_halves_shared_accesses_conflict_free(isz, CL):
    for name, width, addrs in halves_accesses(isz, CL):
        need, ideal = wavefronts(addrs, width)
        assert need == ideal, f"{name}: {need} wavefronts, {ideal} without conflicts"


@pytest.mark.parametrize("LB", [12, 13])
def test_rht_tile_layouts_are_permutations(LB):
    """Each transpose writes every element of the tile once and reads every
    element once; the epilogue's output indices cover the part once."""
    n = 1 << LB
    NT = 1 << (LB - 4)
    shfl12 = LB == 13
    prev, p = 0, 4
    while p - 4 < (8 if shfl12 else LB - 4):
        pp = min(p, LB - 4)
        st = sorted(swz((t & ((1 << prev) - 1)) | ((t >> prev) << (prev + 4)) + (j << prev))
                    for t in range(NT) for j in range(16))
        if shfl12 and pp == 8:
            ld = sorted(swz(elem12(t, 0) + (j << pp)) for t in range(NT) for j in range(16))
        else:
            ld = sorted(swz((t & ((1 << pp) - 1)) | ((t >> pp) << (pp + 4)) + (j << pp))
                        for t in range(NT) for j in range(16))
        assert st == list(range(n)) and ld == list(range(n))
        prev, p = pp, p + 4
    idx = sorted(out_idx(t, j, LB) for t in range(NT) for j in range(16))
    assert idx == list(range(n))


# ---- rht_halves_kernel: rows of 16384 (one CTA) and 32768 (2-CTA cluster) ----

def _stages(x, bits):
    """Butterfly stages h = 2^0 .. 2^(bits-1) over the last axis, in order:
    lower a + b, upper a - b (float64, the kernel's and the reference's order)."""
    import numpy as np
    x = np.array(x, np.float64)
    n = x.shape[-1]
    for b in range(bits):
        h = 1 << b
        y = x.reshape(x.shape[:-1] + (n // (2 * h), 2, h))
        a, c = y[..., 0, :].copy(), y[..., 1, :].copy()
        y[..., 0, :], y[..., 1, :] = a + c, a - c
        x = y.reshape(x.shape)
    return x


def _halves_model(row, CL):
    """Output of rht_halves_kernel's butterflies for one row (before scaling),
    following its register map: after a part's bits 0..12, thread t register j
    holds element elem12(t, j) of the part; bit 13 pairs register j of the
    CTA's two parts; CL = 2: bit 14 pairs register j of the two CTAs, CTA 0
    keeping its sums and receiving CTA 1's, CTA 1 keeping its differences and
    receiving CTA 0's; sums go to out_sum(j), differences to out_dif(j)."""
    import numpy as np
    HALF = 8192
    parts = _stages(np.asarray(row).reshape(-1, HALF), 13)   # each part, bits 0..12
    regs = {}
    for rank in range(CL):
        xa = np.empty((512, 16)); x = np.empty((512, 16))
        for t in range(512):
            for j in range(16):
                xa[t, j] = parts[2 * rank][elem12(t, j)]
                x[t, j] = parts[2 * rank + 1][elem12(t, j)]
        regs[rank] = (xa + x, xa - x)                           # bit 13
    out = np.full(CL * 2 * HALF, np.nan)
    for rank in range(CL):
        if CL == 2:
            own = regs[rank][1] if rank else regs[rank][0]
            got = regs[rank ^ 1][1] if rank else regs[rank ^ 1][0]   # what the partner pushed
            lo, hi = (got, own) if rank else (own, got)
            s, d = lo + hi, lo - hi                               # bit 14
        else:
            s, d = regs[rank]
        for t in range(512):
            for j in range(16):
                e = elem12(t, j)
                out[(0 if CL == 1 else rank * HALF) + e] = s[t, j]
                out[(HALF if CL == 1 else 2 * HALF + rank * HALF) + e] = d[t, j]
    return out


@pytest.mark.parametrize("n,CL", [(16384, 1), (32768, 2)])
def test_halves_kernel_data_flow(n, CL):
    """Every output column written once, bit-identical to the whole-row
    butterflies in stage order."""
    import numpy as np
    rng = np.random.RandomState(n)
    row = rng.standard_normal(n)
    got = _halves_model(row, CL)
    assert not np.isnan(got).any()
    ref = _stages(row, n.bit_length() - 1)
    assert np.array_equal(got.view(np.uint64), ref.view(np.uint64))
