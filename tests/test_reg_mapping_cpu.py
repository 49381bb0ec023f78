"""CPU: the register-operand kernel's operand mapping (csrc/gemm_reg_kernel.cuh), restated in numpy and checked
against exact integer products, without a GPU.

The kernel walks K in double steps of 64 and gives lane (g, t) of a warp codes 16t .. 16t+15 of a channel row
(expanded from one panel word by two byte-permute lookups per register pair) and bytes 16t .. 16t+15 of a token row
(one 16-byte load); MMA h of the double step uses the half 16t + 8h .. 16t + 8h + 7. This test builds those lane
registers from the oracle's panel bytes with the kernel's word index, shift, mask and lookup table, feeds them
through the PTX fragment layout of mma.m16n8k32 (.s8 A row-major 16 x 32, B column-major 32 x 8, D 16 x 8 INT32),
and requires the sums to equal the exact dot products - the K-order argument the kernel rests on."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from kea_kernels import formats
from kea_kernels.binary import bits

SIGN_TABLE, TERNARY_TABLE = 0x000001FF, 0x00FF0100   # byte-permute tables of the expanders (nibble -> int8 byte)


def _lookup4(table: int, sel: int) -> np.ndarray:
    """prmt(table, 0, sel): the low four selector nibbles each pick a byte of (table, 0) -> 4 int8 values."""
    tb = [(table >> (8 * i)) & 0xFF for i in range(4)] + [0, 0, 0, 0]
    return np.array([tb[(sel >> (4 * j)) & 0x7] for j in range(4)], dtype=np.uint8).view(np.int8)


def _panel_word(pan: np.ndarray, wbits: int, kb_total: int, n: int, w: int) -> int:
    """Word w (over the row's k-blocks, sub-blocks and four words) of channel row n: [tile][kb][sub][4][128][4]."""
    tile_words = kb_total * 4 * wbits * 128
    idx = (n >> 7) * tile_words + w * 128 + (n & 127)
    return int(pan.view(np.uint32)[idx])


def _lane_a(pan, wbits, kb_total, n, s, t, h) -> np.ndarray:
    """The 8 int8 weights lane t holds for MMA h of double step s of channel row n (registers 0 and 2 of its row)."""
    if wbits == 1:
        word = _panel_word(pan, 1, kb_total, n, 2 * s + t // 2)
        sel = (word >> (2 * (t % 2) + h)) & 0x11111111
        table = SIGN_TABLE
    else:
        word = _panel_word(pan, 2, kb_total, n, 4 * s + t)
        sel = (word >> (2 * h)) & 0x33333333
        table = TERNARY_TABLE
    return np.concatenate([_lookup4(table, sel), _lookup4(table, sel >> 16)])


def _mma_m16n8k32(a_regs: dict, b_regs: dict) -> np.ndarray:
    """D[16][8] = A[16][32] B[32][8] from per-lane registers, with the PTX fragment layout of m16n8k32 (.s8):
    lane (g, t): A regs 0 / 1 / 2 / 3 = A[g][4t..], A[g+8][4t..], A[g][16+4t..], A[g+8][16+4t..]; B regs 0 / 1 =
    B[4t..][g], B[16+4t..][g]."""
    a = np.zeros((16, 32), dtype=np.int64)
    b = np.zeros((32, 8), dtype=np.int64)
    for lane in range(32):
        g, t = lane // 4, lane % 4
        r0, r1, r2, r3 = a_regs[lane]
        a[g, 4 * t:4 * t + 4], a[g + 8, 4 * t:4 * t + 4] = r0, r1
        a[g, 16 + 4 * t:20 + 4 * t], a[g + 8, 16 + 4 * t:20 + 4 * t] = r2, r3
        b0, b1 = b_regs[lane]
        b[4 * t:4 * t + 4, g], b[16 + 4 * t:20 + 4 * t, g] = b0, b1
    return a @ b


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("k", [64, 256, 1024])
@pytest.mark.parametrize("c0", [0, 48, 112])   # a 16-channel group at any offset inside a 128-row panel tile
def test_lane_registers_give_the_exact_products(wbits, k, c0):
    n, rows = 128, 8
    g = torch.Generator().manual_seed(wbits * 1000 + k + c0)
    if wbits == 1:
        w = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
        codes = bits.pack_signs(w).numpy()
    else:
        u = torch.rand(n, k, generator=g)
        w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
        codes = formats.pack_ternary(w).numpy()
    w = w.numpy().astype(np.int64)
    q = torch.randint(-127, 128, (rows, k), generator=g, dtype=torch.int8).numpy()
    pan = oracle.panels(codes, wbits, n, k)
    kb_total = -(-k // 128)

    acc = np.zeros((16, 8), dtype=np.int64)
    for s in range(k // 64):
        for h in range(2):
            a_regs, b_regs = {}, {}
            for lane in range(32):
                gg, t = lane // 4, lane % 4
                lo = _lane_a(pan, wbits, kb_total, c0 + gg, s, t, h)        # channel row g
                hi = _lane_a(pan, wbits, kb_total, c0 + gg + 8, s, t, h)    # channel row g + 8
                a_regs[lane] = (lo[:4], hi[:4], lo[4:], hi[4:])
                seg = q[gg, 64 * s + 16 * t + 8 * h: 64 * s + 16 * t + 8 * h + 8].astype(np.int64)
                b_regs[lane] = (seg[:4], seg[4:])
            acc += _mma_m16n8k32(a_regs, b_regs)
    want = w[c0:c0 + 16] @ q.astype(np.int64).T
    assert np.array_equal(acc, want)


def test_lookup_tables_expand_codes():
    # 1-bit: code 0 -> -1, 1 -> +1; ternary field 0 -> 0, 1 -> +1, 2 -> -1 (the export's encodings)
    assert _lookup4(SIGN_TABLE, 0x1010).tolist() == [-1, 1, -1, 1]
    assert _lookup4(TERNARY_TABLE, 0x0210).tolist() == [0, 1, -1, 0]
