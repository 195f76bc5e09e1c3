"""Bit-packing of 2/3/4-bit codes along the last dim (CUDA).

Same API and byte layout as the reference ``akv/bitpack.py``:
  * uint4: even index -> high nibble, odd index -> low nibble (:13-30)
  * uint3: 8 codes -> 24-bit word c0<<21 | ... | c7 -> 3 bytes big-endian (:35-68)
  * uint2: 4 codes per byte, first code in the top two bits (:73-90)
  * rows are right-padded with zero codes to the pack group; other widths pass
    through unchanged (:95-114).
The work runs in ``libakv_sm100.so`` (akv_pack_codes / akv_unpack_codes).
"""
from __future__ import annotations

import torch

from . import _C


def packed_width(dim: int, bits: int) -> int:
    if bits == 4:
        return (dim + 1) // 2
    if bits == 3:
        return (dim + 7) // 8 * 3
    if bits == 2:
        return (dim + 3) // 4
    return dim


def _pack(indices: torch.Tensor, bits: int) -> torch.Tensor:
    _C.require_cuda(indices)
    x = indices if indices.dtype == torch.uint8 else indices.to(torch.uint8)
    x = x.contiguous()
    D = x.shape[-1]
    rows = x.numel() // D if D else 0
    out = torch.empty(x.shape[:-1] + (packed_width(D, bits),), dtype=torch.uint8, device=x.device)
    if rows:
        _C.check(_C.load().akv_pack_codes(x.data_ptr(), rows, D, bits, out.data_ptr(), _C.stream_of(x)),
                 "akv_pack_codes")
    return out


def _unpack(packed: torch.Tensor, bits: int, orig_dim: int) -> torch.Tensor:
    _C.require_cuda(packed)
    p = packed.contiguous()
    if p.dtype != torch.uint8:
        raise TypeError("packed codes must be uint8")
    if p.shape[-1] != packed_width(orig_dim, bits):
        raise ValueError(f"packed width {p.shape[-1]} does not match orig_dim={orig_dim} at {bits} bits")
    rows = p.numel() // p.shape[-1] if p.shape[-1] else 0
    out = torch.empty(p.shape[:-1] + (orig_dim,), dtype=torch.uint8, device=p.device)
    if rows:
        _C.check(_C.load().akv_unpack_codes(p.data_ptr(), rows, orig_dim, bits, out.data_ptr(), _C.stream_of(p)),
                 "akv_unpack_codes")
    return out


def pack_uint4(indices: torch.Tensor) -> torch.Tensor:
    return _pack(indices, 4)


def unpack_uint4(packed: torch.Tensor, orig_dim: int) -> torch.Tensor:
    return _unpack(packed, 4, orig_dim)


def pack_uint3(indices: torch.Tensor) -> torch.Tensor:
    return _pack(indices, 3)


def unpack_uint3(packed: torch.Tensor, orig_dim: int) -> torch.Tensor:
    return _unpack(packed, 3, orig_dim)


def pack_uint2(indices: torch.Tensor) -> torch.Tensor:
    return _pack(indices, 2)


def unpack_uint2(packed: torch.Tensor, orig_dim: int) -> torch.Tensor:
    return _unpack(packed, 2, orig_dim)


def pack(indices: torch.Tensor, bits: int) -> torch.Tensor:
    """Pack indices at the given bit width (8-bit / other widths pass through)."""
    if bits in (2, 3, 4):
        return _pack(indices, bits)
    return indices


def unpack(packed: torch.Tensor, bits: int, orig_dim: int) -> torch.Tensor:
    if bits in (2, 3, 4):
        return _unpack(packed, bits, orig_dim)
    return packed


def packed_bytes(codes: torch.Tensor, bits: int) -> int:
    """Bytes after packing ``codes`` (reference bitpack.py:117-120), from the shape alone."""
    D = codes.shape[-1]
    rows = codes.numel() // D if D else 0
    if bits in (2, 3, 4):
        return rows * packed_width(D, bits)
    return codes.element_size() * codes.numel()
