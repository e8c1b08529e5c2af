"""CPU tests of the LDLQ chain engine's scheduler (kquant_b200.exl3_encoder_backend._chain_traverse).

The launch function is replaced by a recorder and the matrices are meta tensors,
so only the host logic runs: every chain walks its 16-row steps in the backward
buffer order of kquant/exl3_encoder_backend.py:389-505 exactly once, every launch
holds at most KQ_CHAIN_MAX_ITEMS items of one context and either one wave
(2 x SMs tiles) or a nearly full double wave (up to 4 x SMs tiles, two tile pairs
per CTA), and the buffer-end feedback updates happen after a buffer's last step,
on the chain's own columns.
"""
import torch

from kquant_b200 import _native
from kquant_b200 import exl3_encoder_backend as be


def _member(k, n, ctx=128, rate=3, buffer_rows=128):
    """A chain member without device state: meta tensors and a dummy label table per K."""
    m = object.__new__(be._ChainMember)
    m.k, m.n = k, n
    m.W = torch.empty((k, n), device="meta")
    m.P = torch.empty((k, n), device="meta")
    m.E = torch.empty((k, n), device="meta")
    m.wq = torch.empty((k, n), device="meta")
    m.L = torch.empty((k, k), device="meta")
    m.enc = torch.empty((k // 16, n // 16, 256), dtype=torch.int16, device="meta")
    m.buffer_rows = buffer_rows
    m.tf32 = False
    m.rate = rate
    m.ctx = ctx
    bits = {rate} if isinstance(rate, int) else set(rate[1])
    m.labels = {K: torch.empty(65536, dtype=torch.int16, device="meta") for K in bits}
    m.chain_ok = bits <= {2, 3, 4}
    return m


def _run(monkeypatch, members, sms=148):
    launches = []

    def fake_step(items, ctx, device, max_ctas=0):
        launches.append([(it.size_k, it.size_n, it.r0, it.end, it.tile_col0, it.n_tiles, it.K, ctx) for it in items])

    class _Props:
        multi_processor_count = sms

    monkeypatch.setattr(_native, "ldlq_chain_step", fake_step)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda device: _Props())
    trims = []
    real_advance = be._Chain.advance

    def advance(self):
        r0, end = self.steps[self.pos]
        if r0 == end - self.m.buffer_rows and r0 > 0:
            trims.append((id(self.m), self.tile_col0, r0, end))
        real_advance(self)

    monkeypatch.setattr(be._Chain, "advance", advance)
    be._chain_traverse(members, torch.device("cpu"))
    return launches, trims


def _launch_ms(items, sms=148):
    """Model of a launch's duration on B200 (K3, C=128; measured 1.086 ms at one pair per CTA, 2.06 at two):
    0.99 ms per tile pair of the busiest CTA plus 0.09 ms."""
    pairs = sum((i[5] + 1) // 2 for i in items)
    return 0.99 * -(-pairs // sms) + 0.09


def _filled(t, sms=148):
    """A launch is one wave, or nearly full at p = 2..4 tile pairs per SM."""
    return t <= 2 * sms or any(0.9 * 2 * p * sms <= t <= 2 * p * sms for p in range(2, 5))


def test_triplet_schedule_is_valid_and_packed(monkeypatch):
    gate_up = _member(7168, 4096)
    down = _member(2048, 7168)
    launches, trims = _run(monkeypatch, [gate_up, down])
    seen = {}
    for items in launches:
        assert 1 <= len(items) <= _native.KQ_CHAIN_MAX_ITEMS
        assert _filled(sum(i[5] for i in items))
        assert len({i[7] for i in items}) == 1
        cols = [(i[0], i[1], i[4]) for i in items]
        assert len(cols) == len(set(cols))                      # one step per chain per launch
        for k, n, r0, end, c0, nt, _, _ in items:
            seen.setdefault((k, n, c0), []).append((r0, end))
    # every chain: all k/16 steps, backward over 128-row buffers, each exactly once
    for (k, n, c0), steps in seen.items():
        expect = [(end - 128 + le - 16, end) for end in range(k, 0, -128) for le in range(128, 0, -16)]
        assert steps == expect
    assert len(seen) == 4096 // 16 // 32 + 7168 // 16 // 32
    # 172,032 tiles: the critical path is 448 steps; double waves while the work exceeds one wave per
    # critical-path step put the modelled time below the 582 single waves (681 ms) it took before
    assert sum(sum(i[5] for i in items) for items in launches) == 7168 // 16 * 4096 // 16 + 2048 // 16 * 7168 // 16
    assert len(launches) == 448
    assert sum(_launch_ms(items) for items in launches) <= 640
    # trims: one per chain per buffer except the first rows
    assert len(trims) == (4096 // 512) * (7168 // 128 - 1) + (7168 // 512) * (2048 // 128 - 1)


def test_contexts_never_share_a_launch_and_narrow_tail_chains(monkeypatch):
    a = _member(256, 16 * 40, ctx=128, rate=2)       # 40 tile columns: chains of 32 + 8
    b = _member(512, 16 * 32, ctx=64, rate=4)
    launches, _ = _run(monkeypatch, [a, b], sms=16)
    widths = {i[5] for items in launches for i in items if i[1] == 16 * 40}
    assert widths == {32, 8}
    for items in launches:
        assert len({i[7] for i in items}) == 1
        assert sum(i[5] for i in items) <= 8 * 16 or len(items) == 1


def test_mixed_rate_chains(monkeypatch):
    """n-axis rate maps split chains at K changes; k-axis maps change an item's K per step; one launch may mix
    K (one wave), and every item's K is the map's K at its rows and columns."""
    n_bits = ("n", tuple([2] * 8 + [4] * 8 + [3] * 16))     # 32 tile columns: runs 8 (K2), 8 (K4), 16 (K3)
    k_bits = ("k", tuple([3] * 8 + [2] * 4 + [4] * 4))      # 16 tile rows
    a = _member(256, 512, rate=n_bits)
    b = _member(256, 256, rate=k_bits)
    launches, _ = _run(monkeypatch, [a, b], sms=148)
    assert any(len({i[6] for i in items}) > 1 for items in launches)
    for items in launches:
        assert sum(i[5] for i in items) <= 8 * 148
        start = 0
        for size_k, size_n, r0, end, c0, nt, K, ctx in items:
            assert start % 2 == 0
            start += nt
            if size_n == 512:
                assert len(set(n_bits[1][c0:c0 + nt])) == 1 and K == n_bits[1][c0]
            else:
                assert K == k_bits[1][r0 // 16]
    cols = sorted({(i[4], i[5]) for items in launches for i in items if i[1] == 512})
    assert cols == [(0, 8), (8, 8), (16, 16)]


def test_k_axis_prefix_trie_forks(monkeypatch):
    """The k-axis candidate trie on the chain engine (host logic only): every candidate ends in one leaf, every
    step a member runs uses a K that all of the member's candidates map to at those rows, and every chain
    lineage covers all k/16 steps."""
    import contextlib

    k, n = 512, 256
    runs = []

    def fake_item(self):
        r0, _ = self.steps[self.pos]
        runs.append((id(self.m), self.tile_col0, r0, self.K))
        return None

    class _Props:
        multi_processor_count = 148

    monkeypatch.setattr(be._Chain, "item", fake_item)
    monkeypatch.setattr(_native, "ldlq_chain_step", lambda items, ctx, device, max_ctas=0: None)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda device: _Props())
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(be, "get_quant_stream", lambda d: None)
    monkeypatch.setattr(be, "_sync", lambda devices: None)
    monkeypatch.setattr(be, "_labels_for", lambda device, bits, kind, lut: torch.empty(65536, device="meta"))
    nt = k // 16
    maps = [tuple([3] * nt),
            tuple([2] * 8 + [4] * 8 + [3] * 16),          # differs in the top two buffers
            tuple([4] * 8 + [2] * 8 + [3] * 16),
            tuple([3] * 8 + [2] * 4 + [4] * 4 + [3] * 16)]  # differs only in the second buffer
    args = [{"K": 3, "devices": ["meta"], "mixed_rate_axis": "k", "mixed_tile_bits": m, "tailbite_context": 128}
            for m in maps]
    W = torch.empty((2, k, n), device="meta")
    Ls = torch.empty((2, k, k), device="meta")
    wq, enc = be.ldlq_mixed_k_candidates_prefix_reuse(W, Ls, [args, args[:2]])
    assert wq.shape == (6, k, n) and enc.shape == (6, k // 16, n // 16, 256)
    by_member = {}
    for mid, c0, r0, K in runs:
        by_member.setdefault(mid, []).append((c0, r0, K))
    # members that ran steps: each step's K is one of the candidate maps' K at that row
    for steps in by_member.values():
        for c0, r0, K in steps:
            assert K in {m[r0 // 16] for m in maps}
    # each chain column range: the rows run by its lineage cover all k/16 steps at least once per leaf path
    rows_per_col = {}
    for mid, c0, r0, K in runs:
        rows_per_col.setdefault(c0, set()).add(r0)
    assert all(rows == set(range(0, k, 16)) for rows in rows_per_col.values())
    # the shared bottom buffers ran once per source (no forks below the top two buffers)
    bottom = [r for r in runs if r[2] >= 256]
    assert len(bottom) == 2 * (n // 16 // 32 or 1) * (256 // 16)


def test_odd_runs_stay_pair_aligned(monkeypatch):
    """Odd-length K runs along n (single tile columns) never leave two odd items in a mixed-K launch."""
    bits = ("n", tuple([2, 3, 4, 3, 2, 4, 4, 4] * 4))        # runs of length 1 and 3
    a = _member(256, 512, rate=bits)
    launches, _ = _run(monkeypatch, [a], sms=148)
    for items in launches:
        if len({i[6] for i in items}) > 1:
            starts, at = [], 0
            for i in items:
                starts.append(at)
                at += i[5]
            assert all(x % 2 == 0 for x in starts)
    cols = {}
    for items in launches:
        for i in items:
            cols.setdefault((i[4], i[5]), []).append(i[2])
    assert all(len(r) == 256 // 16 for r in cols.values())


def test_mixed_k_slice_refills_after_dropping_odd_chains(monkeypatch):
    """A configs[2]-like slice (4 experts, per-tensor K in {2,3,4}, n-axis odd runs): every mixed launch is
    pair-aligned and fits two same-K pairs per SM; the schedule stays near the modelled lower bound."""
    import bench
    rates = bench.layer_rates()
    members = []
    for e in range(4):
        for (k, n), K in zip(((7168, 2048), (7168, 2048), (2048, 7168)), rates[e]):
            members.append(_member(k, n, rate=K))
    # two n-axis mixed-rate members with odd runs of one K
    members.append(_member(2048, 1024, rate=("n", (2,) * 3 + (4,) * 3 + (3,) * 58)))
    members.append(_member(2048, 1024, rate=("n", (4,) * 5 + (2,) * 5 + (3,) * 54)))
    launches, _ = _run(monkeypatch, members)
    total = sum(it[5] for L in launches for it in L)
    assert total == sum((m.k // 16) * (m.n // 16) for m in members)
    for L in launches:
        assert _filled(sum(it[5] for it in L))
        if len({it[6] for it in L}) > 1:
            starts = [sum(it[5] for it in L[:i]) for i in range(len(L))]
            assert all(s % 2 == 0 for s in starts)
            pairs = {}
            for it in L:
                pairs[it[6]] = pairs.get(it[6], 0) + (it[5] + 1) // 2
            tot = sum(pairs.values())
            assert any(sum(-(-p // m) for p in pairs.values()) <= 148 for m in range(max(1, -(-tot // 148)), 5))
    # throughput bound: four pairs per SM, 0.99 ms per pair per SM
    assert sum(_launch_ms(L) for L in launches) <= 1.08 * (0.99 * total / (2 * 148) + 0.09 * total / (8 * 148))
