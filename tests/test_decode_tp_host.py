"""Host mirror of the tensor-parallel decode step kernel's work plan
(csrc/decode_tp.cu): for the shapes it serves, every weight row is owned by
exactly one CTA per phase, the producer and the consumers walk the same slot
sequence, every slot's bytes fit its 16 KB, every TMA coordinate lies inside
its tensor, the attention plan gives at most one unit per CTA and covers every
cache position once, and the scratch regions fit the staging buffer.  CPU only."""
import pytest

SMS = 148
SLOT, MAX_SLOTS, TOK, GRAN, MAX_GRAN, HD, POS, MAXG = 16384, 12, 8, 8, 16, 128, 64, 8
SMEM_LIMIT = 232448


def gran_range(ng, c, C):
    return ng * c // C, ng * (c + 1) // C


def phase_range(name, N, c, C):
    """Granules of CTA c (the step kernel's gate/up granules hold 4 gate rows
    and the 4 up rows of the same features, so any granule split works)."""
    return gran_range(N // GRAN, c, C)


def kb_per_stage(g, nkb):
    return min(16 // g, nkb)


def copies(n):
    """(first block, depth) of the copies of an n-block stage: 8, 4, 2, 1 blocks, largest first."""
    out, q = [], 0
    while q < n:
        r = n - q
        d = 8 if r >= 8 else 4 if r >= 4 else 2 if r >= 2 else 1
        out.append((q, d))
        q += d
    return out


def att_plan(pairs, L, C):
    sp = max(1, C // pairs)
    sp = min(sp, (L + POS - 1) // POS)
    ch = (L + sp - 1) // sp
    ch = (ch + POS - 1) // POS * POS
    sp = (L + ch - 1) // ch
    return sp, ch


def phases(H, Hq, Hkv, I):
    # (name, N, K)
    return [("qkv", (Hq + 2 * Hkv) * HD, H), ("att", 0, 0), ("o", H, Hq * HD),
            ("gu", 2 * I, H), ("dn", H, I)]


def schedule(c, C, H, Hq, Hkv, I, M, L, max_seq):
    """Slots of CTA c for one layer: (phase, bytes, [tma boxes (x, y, rows, tensor rows)])."""
    out = []
    sp, ch = att_plan(M * Hkv, L, C)
    for name, N, K in phases(H, Hq, Hkv, I):
        if name == "att":
            if c < M * Hkv * sp:
                pair, split = divmod(c, sp)
                b, kvh = divmod(pair, Hkv)
                start, end = split * ch, min(split * ch + ch, L - 1)
                for t0 in range(start, end, POS):
                    row = (b * Hkv + kvh) * max_seq + t0
                    for _ in range(2):
                        out.append((name, SLOT, [(0, row, POS), (64, row, POS)],
                                    M * Hkv * max_seq, 128))
            continue
        lo, hi = phase_range(name, N, c, C)
        g = hi - lo
        if g == 0:
            continue
        nkb = K // 64
        kbs = kb_per_stage(g, nkb)
        assert g * kbs * 1024 <= SLOT
        for kb0 in range(0, nkb, kbs):
            n = min(kbs, nkb - kb0)
            cps = copies(n)
            # copies of 8/4/2/1 K blocks, all g granules: x = first K block of the copy
            boxes = [(kb0 + q, lo * GRAN, g * GRAN, d) for q, d in cps]
            spans = [(q * g * 1024, (q + d) * g * 1024) for q, d in cps]
            assert sum(d for _, d in cps) == n and all(d in (1, 2, 4, 8) for _, d in cps)
            for a, b in spans:      # inside the slot, no overlap, [K block][row] order
                assert b <= SLOT
            assert spans[0][0] == 0
            assert all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
            # the consumer's address of (K block j, granule gi) lies in the copy holding j
            for j in range(n):
                for gi in range(g):
                    off = (j * g + gi) * 1024
                    q, d = next((q, d) for q, d in cps if q <= j < q + d)
                    assert spans[cps.index((q, d))][0] <= off < spans[cps.index((q, d))][1]
            out.append((name, g * n * 1024, boxes, N, K))
    return out


CASES = [  # (label, H, Hq, Hkv, I, M, L, max_seq)
    ("8B TP2", 4096, 16, 4, 6144, 8, 1152, 2048),
    ("8B TP4", 4096, 8, 2, 3072, 8, 1152, 2048),
    ("8B TP8", 4096, 4, 1, 1536, 8, 1152, 2048),
    ("8B TP8 B1 long", 4096, 4, 1, 1536, 1, 8000, 8192),
    ("8B TP8 B3 L2", 4096, 4, 1, 1536, 3, 2, 2048),
    ("tiny TP1", 512, 4, 1, 1024, 1, 60, 256),
    ("tiny8 TP1", 512, 8, 2, 1024, 1, 45, 256),
]


@pytest.mark.parametrize("label,H,Hq,Hkv,I,M,L,max_seq", CASES)
def test_plan_covers_rows_once_and_stays_in_bounds(label, H, Hq, Hkv, I, M, L, max_seq):
    C = SMS
    for name, N, K in phases(H, Hq, Hkv, I):
        if name == "att":
            continue
        ng = N // GRAN
        owned = []
        for c in range(C):
            lo, hi = phase_range(name, N, c, C)
            assert hi - lo <= MAX_GRAN, (label, name, hi - lo)
            owned.extend(range(lo, hi))
        assert owned == list(range(ng)), (label, name)
        assert K % 64 == 0 and N % GRAN == 0
    # attention: units <= C, every old position streamed once, the new one by one split
    sp, ch = att_plan(M * Hkv, L, C)
    assert M * Hkv * sp <= C
    seen = {}
    for c in range(M * Hkv * sp):
        pair, split = divmod(c, sp)
        start, end = split * ch, min(split * ch + ch, L - 1)
        for t in range(start, end):
            seen[(pair, t)] = seen.get((pair, t), 0) + 1
        assert (start <= L - 1 < start + ch) == (split == (L - 1) // ch)
    assert all(v == 1 for v in seen.values())
    assert len(seen) == M * Hkv * (L - 1)
    # slots: bytes and TMA boxes inside their tensors (x a multiple of 64 elements)
    for c in range(C):
        for name, nbytes, boxes, rows, cols in schedule(c, C, H, Hq, Hkv, I, M, L, max_seq):
            assert 0 < nbytes <= SLOT
            for box in boxes:
                if name != "att":
                    kb, y, r, dep = box
                    assert kb + dep <= cols // 64 and y + r <= rows   # exact, no overrun
                    assert r <= 256 and dep <= 256                   # TMA box limits
                else:
                    x, y, r = box
                    assert x % 64 == 0 and x + 64 <= cols
                    assert y < rows   # a tile may run past the head: TMA fills zeros


@pytest.mark.parametrize("label,H,Hq,Hkv,I,M,L,max_seq", CASES)
def test_shared_memory_and_exchange_sizes(label, H, Hq, Hkv, I, M, L, max_seq):
    kmax = max(H, Hq * HD, I)
    x_stride = kmax * 2 + 16
    # warp partials, bf16 exchange partials, the outputs' squares
    red = 4 * MAX_GRAN * GRAN * TOK * 4 + MAX_GRAN * GRAN * TOK * 2 + MAX_GRAN * GRAN * TOK * 4
    # attention scratch, and the per-pair merge's weights and products after q
    MAX_SPLITS = 256
    att = MAXG * HD * 2 + max(4 * MAXG * HD + 4 * MAXG * 2 + 2 * HD + MAXG + 1,
                              2 * MAX_SPLITS * MAXG + MAXG + MAXG * HD + MAX_SPLITS) * 4
    sp, ch = att_plan(M * Hkv, L, SMS)
    assert sp <= MAX_SPLITS
    # a split's slice of the merge: splits x slice products fit the scratch
    G = Hq // Hkv
    per = -(-G * HD // sp)
    assert sp * per <= MAXG * HD + MAX_SPLITS
    # eight token rows, the RMSNorm weight row, the per-CTA sums of squares
    x_bytes = -(-max((TOK + 1) * x_stride + SMS * TOK * 4, red, att) // 1024) * 1024
    fixed = x_bytes + 1024 + 2 * MAX_SLOTS * 8 + 5 * TOK * 4 + 8
    # bulk copies: 16-byte aligned rows and sizes
    assert x_stride % 16 == 0 and ((TOK + 1) * x_stride) % 16 == 0
    for K in (H, Hq * HD, I):
        assert (K * 2) % 16 == 0
    nslots = min(MAX_SLOTS, (SMEM_LIMIT - fixed) // SLOT)
    assert nslots >= 3, label
    assert nslots * SLOT + fixed <= SMEM_LIMIT
    # A-fragment rows of the staging buffer stay bank-conflict free: the row
    # stride is 16 bytes past a multiple of 128
    assert x_stride % 128 == 16
    # the inbox: [2 parities][8 sources][H rows][4 token pairs] 8-byte words
    # inside a communicator created with max_cols = H
    inbox = 2 * 8 * H * 4 * 8
    comm_data = 2 * 8 * (H // 64) * (64 * 16 // 2) * 8
    assert inbox <= comm_data


def test_producer_and_consumers_walk_the_same_slots():
    """Both sides derive the slot sequence from the same functions; here the
    consumer's count (project: one slot per stage; attention: two per tile)
    equals the producer's for every CTA of the 8B TP8 step over 36 layers."""
    H, Hq, Hkv, I, M, L, max_seq = 4096, 4, 1, 1536, 8, 1152, 2048
    C = SMS
    sp, ch = att_plan(M * Hkv, L, C)
    for c in range(C):
        prod = len(schedule(c, C, H, Hq, Hkv, I, M, L, max_seq)) * 36
        cons = 0
        for name, N, K in phases(H, Hq, Hkv, I):
            if name == "att":
                if c < M * Hkv * sp:
                    pair, split = divmod(c, sp)
                    start, end = split * ch, min(split * ch + ch, L - 1)
                    cons += 2 * len(range(start, end, POS))
                continue
            lo, hi = phase_range(name, N, c, C)
            if hi > lo:
                nkb = K // 64
                cons += -(-nkb // kb_per_stage(hi - lo, nkb))
        assert prod == cons * 36


def test_gate_up_granules_hold_whole_features():
    """ops.gate_up_granules4: from q3_gemm's 8-row gate/up interleave to the step
    kernel's granules of 4 gate rows then the same 4 features' up rows."""
    import torch
    from q3vl import layout
    from q3vl.ops import gate_up_granules4
    I, H = 96, 3
    gate = torch.randn(I, H)
    up = torch.randn(I, H)
    w4 = gate_up_granules4(layout.interleave_gate_up(gate, up))
    assert w4.shape == (2 * I, H)
    for j in range(2 * I // GRAN):
        assert torch.equal(w4[8 * j:8 * j + 4], gate[4 * j:4 * j + 4])
        assert torch.equal(w4[8 * j + 4:8 * j + 8], up[4 * j:4 * j + 4])
