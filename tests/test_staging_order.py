"""A CPU model of the activation-staging loops of the decode GEMVs (csrc/w4a16.cu `stage_x`,
csrc/w8a16.cu) in their batched form: each thread issues the loads of kBatch loop iterations before
it stores any of them.

The batched loop must stage the same items as the one-at-a-time loop: every item once, each by the
thread that staged it before. The one-row W4A16 path keeps x + residual in registers between the
sum-of-squares pass and the staging, and relies on that. In the W4A16 loop the range check of each
batched iteration must also be the same for all 32 lanes of a warp, because the factored path reduces
each 128-group with warp shuffles. Both properties are index arithmetic, checked here for the row
counts and K slices the kernels take."""

import pytest

KWARPS = 8
KTHR = KWARPS * 32  # consumer threads that stage (both GEMVs)


def one_at_a_time_w4(items: int) -> dict:
    """csrc/w4a16.cu before batching: for (base = tid & ~31; base < items; base += kThr), item base + lane."""
    owner = {}
    for tid in range(KTHR):
        base = tid & ~31
        while base < items:
            i = base + (tid & 31)
            assert i not in owner
            owner[i] = tid
            base += KTHR
    return owner


def batched_w4(items: int, kbatch: int) -> dict:
    """The batched loop: base0 steps by kBatch * kThr; iteration u stages item base0 + u * kThr + lane
    when base0 + u * kThr < items (the same test for every lane of the warp)."""
    owner = {}
    for warp in range(KWARPS):
        for base0 in range(warp * 32, items, kbatch * KTHR):
            for u in range(kbatch):
                in_range = [base0 + u * KTHR < items for _ in range(32)]  # what each lane tests
                assert len(set(in_range)) == 1, "range check differs across the warp"
                if not in_range[0]:
                    continue
                for lane in range(32):
                    i = base0 + u * KTHR + lane
                    assert i < items
                    assert i not in owner
                    owner[i] = warp * 32 + lane
    return owner


def one_at_a_time_w8(items: int) -> dict:
    owner = {}
    for tid in range(KTHR):
        for i in range(tid, items, KTHR):
            assert i not in owner
            owner[i] = tid
    return owner


def batched_w8(items: int, kb: int) -> dict:
    """csrc/w8a16.cu: for (i0 = tid; i0 < items; i0 += kB * kThr8), item i0 + u * kThr8 when < items."""
    owner = {}
    for tid in range(KTHR):
        for i0 in range(tid, items, kb * KTHR):
            for u in range(kb):
                i = i0 + u * KTHR
                if i >= items:
                    break
                assert i not in owner
                owner[i] = tid
    return owner


# W4A16: an item is 8 K values of one row; nblk = staged 256-wide K stages x 32 blocks (a multiple of 32)
@pytest.mark.parametrize("M", [1, 2, 8, 9, 13, 16])
@pytest.mark.parametrize("stages", [1, 2, 3, 6, 35])
@pytest.mark.parametrize("kbatch", [1, 4])
def test_w4a16_batched_staging_keeps_item_owners(M, stages, kbatch):
    items = M * stages * 32
    ref = one_at_a_time_w4(items)
    got = batched_w4(items, kbatch)
    assert len(got) == items
    assert got == ref


# FP8: an item is 4 K values of one row (4 per 16-wide block); nblk = stages x 128 K / 16
@pytest.mark.parametrize("M", [1, 4, 9, 16])
@pytest.mark.parametrize("stages", [1, 3, 12, 70])
@pytest.mark.parametrize("kb", [1, 4])
def test_w8a16_batched_staging_keeps_item_owners(M, stages, kb):
    items = M * stages * (128 // 16) * 4
    ref = one_at_a_time_w8(items)
    got = batched_w8(items, kb)
    assert len(got) == items
    assert got == ref
