"""Host logic of the tcgen05 prefill kernel's schedules (no GPU needed).

`awq_tc_schedule` reports what `launch_gemm_tc` (csrc/awq_gemm_tc.cu) would run: one CTA per
256 x 256 (or 128 x 256) output tile, persistent CTAs, stream-K or split-K.  For stream-K
the kernel builds each CTA's segments on the device (the segment builder at the top of
`gemm_tc_kernel`); `_segments` below restates it, so the test checks the host plan and the
device builder together: every (tile, K step) is computed exactly once, a tile has at most
three parts with distinct slots 0..n-1 that agree on n, and no CTA reaches more than eight
tiles -- the limits the kernel's slot array and segment array are sized for.
"""
from __future__ import annotations

import ctypes

import pytest

BK, BN, SLOTS, MAX_SEG = 64, 256, 3, 8
GRID, PERSISTENT, STREAMK, SPLITK = 0, 1, 2, 3


@pytest.fixture(scope="module")
def lib():
    import awq_b200._lib as L
    return L.load()


def _schedule(lib, M, N, K, sms):
    kind, param = ctypes.c_int(-1), ctypes.c_int(-1)
    rc = lib.awq_tc_schedule(M, N, K, sms, ctypes.byref(kind), ctypes.byref(param))
    assert rc == 0, lib.awq_last_error()
    return kind.value, param.value


def _segments(c, tiles, S, kt, G, tiles_n):
    """CTA c's segments (tile_m, tile_n, k0, k1, idx, n) under stream-K: CTA c < tiles runs
    steps [0, S) of tile c (slot 0); CTA tiles + j shares the tails in linear order."""
    L = kt - S
    G2, TT = G - tiles, tiles * L
    start = lambda j: j * TT // G2

    def cta_of(u):
        j = u * G2 // TT
        if j + 1 < G2 and start(j + 1) <= u:
            j += 1
        return j

    if c < tiles:
        jf, jl = cta_of(c * L), cta_of(c * L + L - 1)
        return [(c // tiles_n, c % tiles_n, 0, S, 0, jl - jf + 2)]
    j = c - tiles
    u, u1, out = start(j), start(j + 1), []
    while u < u1:
        t = u // L
        tb = t * L
        e = min(u1, tb + L)
        jf, jl = cta_of(tb), cta_of(tb + L - 1)
        out.append((t // tiles_n, t % tiles_n, S + u - tb, S + e - tb, j - jf + 1, jl - jf + 2))
        u = e
    return out


def test_qwen2_prefill_schedules(lib):
    """The schedules of the Qwen2-7B prefill products on a 148-SM B200."""
    assert _schedule(lib, 2048, 37888, 3584, 148) == (PERSISTENT, 8 * 148)   # gate+up
    assert _schedule(lib, 2048, 3584, 18944, 148) == (STREAMK, 232)          # down: 112 tiles
    assert _schedule(lib, 1536, 3584, 18944, 148) == (STREAMK, 175)          # 84 tiles
    assert _schedule(lib, 2048, 3584, 3584, 148) == (GRID, 112)              # o: 56 K steps, too short
    assert _schedule(lib, 24, 3584, 18944, 148) == (SPLITK, 10)              # 14 tiles
    assert _schedule(lib, 300, 768, 1024, 148) == (SPLITK, 2)                # 6 tiles, K / 512 = 2
    assert _schedule(lib, 2048, 4608, 3584, 148)[0] == GRID                  # q/k/v: 144 tiles


@pytest.mark.parametrize("sms", [148, 132, 120])
def test_stream_k_plans_cover_every_step_once(lib, sms):
    seen = 0
    for M in list(range(129, 4097, 127)) + [1024, 1536, 2048, 2560, 3072]:
        for K, N in [(18944, 3584), (18944, 3360), (18944, 4608), (3584, 3584), (3584, 4608),
                     (3584, 18944), (8192, 1024), (2048, 2304), (1024, 8192)]:
            kind, S = _schedule(lib, M, N, K, sms)
            if kind != STREAMK:
                continue
            seen += 1
            bm = 256 if M > 128 else 128
            tiles_n = -(-N // BN)
            tiles = -(-M // bm) * tiles_n
            kt = K // BK
            assert 2 * tiles >= sms and tiles < sms and kt // 2 <= S < kt, (M, N, K, S)
            cover, parts = {}, {}
            for c in range(sms):
                segs = _segments(c, tiles, S, kt, sms, tiles_n)
                assert 1 <= len(segs) <= MAX_SEG, (M, N, K, c, len(segs))
                for tm, tn, k0, k1, idx, n in segs:
                    assert 0 <= k0 < k1 <= kt and n <= SLOTS
                    t = tm * tiles_n + tn
                    parts.setdefault(t, []).append((idx, n))
                    for k in range(k0, k1):
                        cover[(t, k)] = cover.get((t, k), 0) + 1
            assert len(cover) == tiles * kt and set(cover.values()) == {1}, (M, N, K)
            for t, ps in parts.items():
                n = ps[0][1]
                assert all(p[1] == n for p in ps) and sorted(p[0] for p in ps) == list(range(n)), (t, ps)
    assert seen > 0


def test_schedule_rejects_bad_arguments(lib):
    kind, param = ctypes.c_int(), ctypes.c_int()
    assert lib.awq_tc_schedule(0, 256, 64, 148, ctypes.byref(kind), ctypes.byref(param)) != 0
    assert lib.awq_tc_schedule(16, 256, 100, 148, ctypes.byref(kind), ctypes.byref(param)) != 0
    assert lib.awq_tc_schedule(16, 256, 64, 0, ctypes.byref(kind), ctypes.byref(param)) != 0
    assert lib.awq_tc_schedule(16, 256, 64, 148, None, ctypes.byref(param)) != 0
