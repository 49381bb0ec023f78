"""CPU: the export-code layouts (the reference's tests/test_formats.py:14-59, restated against this package)."""
from __future__ import annotations

import pytest
import torch

from kea_kernels import formats
from kea_kernels.binary import bits


def test_binary_codes_round_trip_and_layout():
    signs = torch.where(torch.rand(5, 21) < 0.5, -1, 1).to(torch.int8)
    packed = bits.pack_signs(signs)
    assert packed.dtype == torch.uint8 and packed.shape == (5, 3)
    assert torch.equal(bits.unpack_signs(packed, 21), signs)
    one = torch.full((1, 8), -1, dtype=torch.int8)
    one[0, 3] = 1
    assert bits.pack_signs(one).tolist() == [[1 << 3]]


def test_binary_codes_reject_tail_bits_and_bad_signs():
    codes = torch.zeros(2, 2, dtype=torch.uint8)
    codes[0, 1] = 0x80
    with pytest.raises(ValueError, match="tail"):
        bits.unpack_bits(codes, 12)
    with pytest.raises(ValueError):
        bits.pack_signs(torch.zeros(2, 3, dtype=torch.int8))
    with pytest.raises(ValueError):
        bits.unpack_bits(codes, 20)


def test_dense_weight_is_sign_times_row_scale():
    signs = torch.tensor([[1, -1, 1], [-1, -1, 1]], dtype=torch.int8)
    w = bits.dense_weight(bits.pack_signs(signs), torch.tensor([0.5, 2.0]), 3)
    assert torch.equal(w, torch.tensor([[0.5, -0.5, 0.5], [-2.0, -2.0, 2.0]], dtype=torch.float64))


def test_ternary_codes_round_trip_and_layout():
    codes = torch.randint(-1, 2, (4, 13), dtype=torch.int8)
    packed = formats.pack_ternary(codes)
    assert packed.shape == (4, 4)
    assert torch.equal(formats.unpack_ternary(packed, 13), codes)
    assert formats.pack_ternary(torch.tensor([[0, 1, -1, 1]], dtype=torch.int8)).tolist() == [[0b01_10_01_00]]


def test_ternary_codes_reject_the_unused_pattern():
    with pytest.raises(ValueError):
        formats.unpack_ternary(torch.tensor([[0b11]], dtype=torch.uint8), 4)
    with pytest.raises(ValueError):
        formats.unpack_ternary(torch.tensor([[0b01_00_00_00]], dtype=torch.uint8), 3)
    with pytest.raises(ValueError):
        formats.pack_ternary(torch.tensor([[2]], dtype=torch.int8))


def test_resident_bytes_counts_storages_once():
    assert bits.resident_bytes(torch.zeros(4), None) == 0   # host tensors do not count
