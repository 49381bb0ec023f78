"""Tile choices of the B200 low-bit GEMM: the M-bucketed split-K dispatch table.

The reference picks an SM120 `DotConfig` from a table of RTX 5090 sweeps (src/kea_kernels/binary/configs.py:16-58). The
B200 kernel has four knobs instead: `tile_m` (tokens per CTA: one or two tcgen05 M = 128 blocks), `tile_n`
(channels per CTA = the tcgen05 N dimension: 32, 64, 128 or 256), `splits` (K split across a thread-block cluster,
reduced exactly in INT32 through distributed shared memory) and `stages` (k128 blocks in flight). The table itself
lives in the C library (`kea_lowbit_choose_config`), so C callers and Python pick the same tiles; selection is a pure
function of (M, N, K, wbits, parts), with no run-time autotuning.
"""
from __future__ import annotations

import dataclasses

from kea_kernels import _lib

SMS = 148


PER_TILE, PAIR, GEMV, SWAP, REG = 0, 1, 2, 3, 4


@dataclasses.dataclass(frozen=True)
class DotConfig:
    """CTA = `tile_m` tokens x `tile_n` channels over 1/`splits` of K, `stages` k128 blocks in flight (the per-tile
    tcgen05 kernel). kernel == PAIR: the persistent CTA-pair kernel, 256 x 256 tiles per pair of SMs (tcgen05
    cta_group::2), walked by at most SMS / 2 pairs, two accumulator buffers in tensor memory. kernel == GEMV: the
    CUDA-core kernel for M <= 16, `tile_n` channels per CTA. kernel == SWAP: the small-M kernel with the operands
    swapped (128 weight rows on the MMA's M axis, every part's `tile_m` tokens on its N axis, K split over a cluster
    of `splits` CTAs). kernel == REG: the small-M register-operand kernel (warp-level MMAs, weights expanded in
    registers), `tile_n` channels x `tile_m` activation rows (tokens x parts) per CTA, K cut into `splits` slices
    among its 8 warps. Passing a PER_TILE config forces those tiles; a SWAP config forces the swap kernel with its
    splits and stages; a REG config the register kernel with its tiles."""
    tile_m: int
    tile_n: int
    splits: int
    stages: int
    kernel: int = PER_TILE

    @property
    def pair(self) -> bool:
        return self.kernel == PAIR

    def label(self) -> str:
        if self.kernel == PAIR:
            return f"pair{self.tile_m}x{self.tile_n}_s{self.stages}"
        if self.kernel == GEMV:
            return f"gemv_n{self.tile_n}"
        if self.kernel == SWAP:
            return f"swap_t{self.tile_m}_c{self.splits}_s{self.stages}"
        if self.kernel == REG:
            return f"reg_r{self.tile_m}_n{self.tile_n}_k{self.splits}"
        return f"m{self.tile_m}_n{self.tile_n}_c{self.splits}_s{self.stages}"

    def validate(self, parts: int = 1) -> None:
        if self.kernel == GEMV:
            if not (1 <= self.tile_m <= 16 and self.tile_n in (8, 16, 32)):
                raise ValueError(f"invalid config {self}")
            return
        if self.kernel == REG:
            cw = 8 // self.splits if self.splits in (1, 2, 4, 8) else 0
            cg = self.tile_n // (16 * cw) if cw and self.tile_n % (16 * cw) == 0 else 0
            if not (self.tile_n in (16, 32, 64, 128) and self.tile_m in (16, 32) and self.stages == 0
                    and (cg, self.tile_m // 8) in ((1, 4), (2, 4), (2, 2), (4, 2)) and self.tile_m // parts >= 1):
                raise ValueError(f"invalid config {self}")
            return
        if self.kernel == SWAP:
            if not (1 <= self.splits <= 16 and 1 <= self.stages <= 8 and self.tile_m % 16 == 0 and self.tile_m >= 0):
                raise ValueError(f"invalid config {self}")
            return
        if not (self.tile_m in (128, 256) and self.tile_n in (32, 64, 128, 256) and 1 <= self.splits <= 16
                and 1 <= self.stages <= 8 and (self.tile_m // 128) * parts * self.tile_n <= 512):
            raise ValueError(f"invalid config {self}")

    def grid(self, m: int, n: int, parts: int = 1) -> tuple[int, int, int]:
        if self.kernel == GEMV:
            return (-(-n // self.tile_n), 1, 1)
        if self.pair:
            tiles = -(-n // self.tile_n) * -(-m // self.tile_m)
            return (2 * min(tiles, SMS // 2), 1, 1)
        if self.kernel == SWAP:
            return (-(-n // 128), -(-m // self.tile_m), self.splits)
        if self.kernel == REG:
            return (-(-n // self.tile_n), -(-m // (self.tile_m // parts)), 1)
        return (-(-n // self.tile_n), -(-m // self.tile_m), self.splits)


def choose(m: int, n: int, k: int, wbits: int = 1, parts: int = 1) -> DotConfig:
    """The configuration the library uses for this shape (the C table)."""
    c = _lib.choose_config(max(m, 0), n, k, wbits, parts)
    return DotConfig(c.tile_m, c.tile_n, c.splits, c.stages, c.kernel)
