"""The index arithmetic of the two-pass NTT schedule (ntt.cu), modelled on CPU.

ntt_pass_kernel keeps 2^R_LOG residues per thread (8 in contiguous passes,
16 in strided ones). Each register group applies up to R_LOG stages, with
twiddle tw[2^(gs0+st) + (prefix << st) + (B << rr) + jw]. This model replays
the same layout and twiddle formulas in Python for a small prime. It checks
that every register layout covers each residue of a sub-transform exactly
once, and that the two passes equal the Longa-Naehrig forward transform. It
also checks that the shared-memory swizzles are bijections and put each
half-warp's 64-bit accesses in 16 distinct bank pairs.
"""
import random

import pytest


def _brev(x, bits):
    return int(format(x, f"0{bits}b")[::-1], 2) if bits else 0


def _prime_and_psi(N):
    q = (1 << 20) // (2 * N) * (2 * N) + 1
    while any(q % p == 0 for p in range(2, int(q ** 0.5) + 1)):
        q += 2 * N
    for g in range(2, q):
        psi = pow(g, (q - 1) // (2 * N), q)
        if pow(psi, N, q) == q - 1:
            return q, psi


def _ln_forward(a, q, tw):
    a, N, t, m = a[:], len(a), len(a), 1
    while m < N:
        t //= 2
        for i in range(m):
            for j in range(2 * i * t, 2 * i * t + t):
                u, v = a[j], a[j + t] * tw[m + i] % q
                a[j], a[j + t] = (u + v) % q, (u - v) % q
        m *= 2
    return a


def _pass(a, q, tw, logN, s_log, strided, r_log):
    N, S, R = 1 << logN, 1 << s_log, 1 << r_log
    T = S // R if S >= R else 1
    ng = (s_log + r_log - 1) // r_log
    stride, gs0 = N >> s_log, (0 if strided else logN - s_log)
    out = a[:]
    for sub in range(N // S):
        prefix = 0 if strided else sub
        gaddr = (lambda r: r * stride + sub) if strided else (lambda r: sub * S + r)
        buf = [out[gaddr(r)] for r in range(S)]
        for gi in range(ng):
            G = min(r_log, s_log - r_log * gi)
            st0, D = r_log * gi, S >> (r_log * gi + G)
            upt, usz = R >> G, 1 << G
            seen = []
            for sub_t in range(T):
                pos = []
                for j in range(upt * usz):
                    u = sub_t + (j // usz) * T
                    pos.append((u // D) * (D << G) + (u % D) + (j % usz) * D)
                x = [buf[r] for r in pos]
                seen += pos
                for uj in range(upt):
                    B = (sub_t + uj * T) // D
                    xu = x[uj * usz:(uj + 1) * usz]
                    for rr in range(G):
                        st, h = st0 + rr, 1 << (G - 1 - rr)
                        idx0 = (1 << (gs0 + st)) + (prefix << st) + (B << rr)
                        for jw in range(1 << rr):
                            w = tw[idx0 + jw]
                            for kk in range(1 << (G - rr)):
                                k = (jw << (G - rr)) + kk
                                if k & h:
                                    continue
                                u0, v0 = xu[k], xu[k + h] * w % q
                                xu[k], xu[k + h] = (u0 + v0) % q, (u0 - v0) % q
                    x[uj * usz:(uj + 1) * usz] = xu
                for j, r in enumerate(pos):
                    buf[r] = x[j]
            assert sorted(seen) == list(range(S)), (s_log, gi)
        for r in range(S):
            out[gaddr(r)] = buf[r]
    return out


@pytest.mark.parametrize("logN", [8, 10, 11])
def test_two_pass_schedule_equals_the_forward_transform(logN):
    N = 1 << logN
    q, psi = _prime_and_psi(N)
    tw = [pow(psi, _brev(k, logN), q) for k in range(N)]
    rng = random.Random(logN)
    a = [rng.randrange(q) for _ in range(N)]
    assert len(set(a)) > N // 2
    s1, s2 = logN // 2, logN - logN // 2
    ref = _ln_forward(a, q, tw)
    # the kernel's choice: 16 residues in strided passes, 8 in contiguous ones
    for r_strided, r_contig in ((4, 3), (3, 3), (4, 4)):
        b = _pass(a, q, tw, logN, s1, True, r_strided)
        assert _pass(b, q, tw, logN, s2, False, r_contig) == ref


def _swizzle(r, r_log):
    h = r >> 4
    if r_log >= 4:
        return h & 15
    return (h & 1) ^ (((h >> 1) & 1) * 6) ^ (((h >> 2) & 1) * 8)


@pytest.mark.parametrize("r_log", [3, 4])
def test_swizzle_is_a_bijection(r_log):
    for S in (16, 32, 64, 128, 256, 512):
        assert sorted(r ^ _swizzle(r, r_log) for r in range(S)) == list(range(S))


def test_sixteen_residue_layouts_are_conflict_free_per_half_warp():
    # thread u of a 256-point block holds r = u + 16 k (first group) and
    # r = 16 u + k (second group); a half-warp is the 16 threads of one block
    for k in range(16):
        for pattern in (lambda u: u + 16 * k, lambda u: 16 * u + k):
            banks = {(pattern(u) ^ _swizzle(pattern(u), 4)) % 16 for u in range(16)}
            assert len(banks) == 16
