"""The roofline arithmetic bench.py reports: algorithmic bytes and FLOPs of
an attention launch, restated by brute force over the rows each query token
attends (its window of up to 128 positions ending at itself, and the
(p + 1) // 128 compressed entries before it)."""

import numpy as np

import bench


def _rows(p):
    win = set(range(max(0, p - 127), p + 1))
    comp = set(range((p + 1) // 128))
    return win, comp


def test_row_bytes():
    # N e4m3 bytes + R bf16 + one UE8M0 scale per 64 NoPE values (the
    # cache's pad byte is not read)
    assert bench.row_bytes_algo(128) == 64 + 128 + 1
    assert bench.row_bytes_algo(512) == 448 + 128 + 7


def test_decode_bytes_and_flops_by_brute_force():
    ctx = np.array([0, 1, 5, 126, 127, 128, 300, 4096, 70000])
    q = bench.Q_PER_SEQ
    heads, d = 64, 128
    rows_total, pairs = 0, 0
    for c in ctx.tolist():
        win_u, comp_u = set(), set()
        for i in range(q):
            w, k = _rows(c + i)
            win_u |= w
            comp_u |= k
            pairs += len(w) + len(k)
        rows_total += len(win_u) + len(comp_u)
    t = len(ctx) * q
    want_bytes = rows_total * bench.row_bytes_algo(d) + 2 * t * heads * d * 2
    assert bench.algorithmic_bytes(ctx, heads, d) == want_bytes
    assert bench.attention_flops(ctx, heads, d) == pairs * heads * 4 * d


def test_prefill_flops_by_brute_force():
    ctx = np.array([0, 256, 1000])
    chunk = 300
    heads, d = 4, 128
    pairs = 0
    for c in ctx.tolist():
        for p in range(c, c + chunk):
            w, k = _rows(p)
            pairs += len(w) + len(k)
    assert bench.prefill_flops(ctx, heads, d, chunk) == float(pairs * heads * 4 * d)
