"""Block-affine (min/max) quantiser for the warm tier, on the GPU.

Drop-in for the reference ``akv/affine_quantizer.py``: same config, same
method names, same returned dict (``codes``, ``scale``, ``zero``,
``orig_dim``, ``bits`` and, with outliers, ``outlier_idx`` / ``outlier_data``)
with the same shapes and bit-identical contents for fp16 input:

  keys   (H, N, D): per-(head, channel) min/max over the N tokens of the call
                    -> scale/zero (H, 1, D)                 (:63-110)
  values (H, N, D): per-(head, token) min/max over D -> scale/zero (H, N, 1)
                                                            (:131-176)
  outliers: top max(1, int(D*fraction)) channels by the mean over heads of
            the per-(head, channel) L2 norm over tokens, kept in fp16 and
            zeroed before quantisation (:75-85, :143-151)

All arithmetic runs in ``libakv_sm100.so`` (``akv_quantize`` /
``akv_dequantize``); inputs must be CUDA fp16 tensors.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _C
from .bitpack import packed_width, pack, unpack


@dataclass
class AffineQuantConfig:
    """Configuration for the block-affine quantiser (reference :25-32)."""
    key_bits: int = 3
    value_bits: int = 3
    group_size: int = 64   # stored for compatibility; the reference does not use it
    packed: bool = True
    outlier_fraction: float = 0.0


def n_outliers(head_dim: int, fraction: float) -> int:
    return max(1, int(head_dim * fraction)) if fraction > 0 else 0


def dict_dest(codes, scale, zero, out_data, out_idx, N: int, D: int, bits: int, n: int, is_key: bool) -> _C.QDest:
    """QDest for the reference dict layout of one call over (H, N, D)."""
    dp = packed_width(D, bits)
    d = _C.QDest()
    d.codes = _C.View(codes.data_ptr(), 0, N * dp, 32 * dp, dp)
    if is_key:
        d.scale = _C.View(scale.data_ptr(), 0, 2 * D, 0, 0)
        d.zero = _C.View(zero.data_ptr(), 0, 2 * D, 0, 0)
    else:
        d.scale = _C.View(scale.data_ptr(), 0, 2 * N, 64, 2)
        d.zero = _C.View(zero.data_ptr(), 0, 2 * N, 64, 2)
    if n:
        d.out_data = _C.View(out_data.data_ptr(), 0, 2 * N * n, 64 * n, 2 * n)
        d.out_idx = _C.View(out_idx.data_ptr(), 0, 0, 0, 0)
    return d


class AffineQuantizer:
    """Block-affine asymmetric quantiser (reference :35-189), CUDA implementation."""

    def __init__(self, config: AffineQuantConfig):
        self.key_bits = config.key_bits
        self.value_bits = config.value_bits
        self.group_size = config.group_size
        self.packed = config.packed
        self.outlier_fraction = config.outlier_fraction

    # ------------------------------------------------------------------
    def _quantize(self, x: torch.Tensor, bits: int, is_key: bool) -> dict:
        _C.require_cuda(x)
        if x.dtype != torch.float16:
            raise TypeError("AffineQuantizer on CUDA takes fp16 tensors (the reference's fp16 arithmetic)")
        if x.dim() != 3:
            raise ValueError("expected (H, N, D)")
        x = x.contiguous()
        H, N, D = x.shape
        n = n_outliers(D, self.outlier_fraction)
        dev = x.device
        codes = torch.empty(H, N, packed_width(D, bits), dtype=torch.uint8, device=dev)
        if is_key:
            scale = torch.empty(H, 1, D, dtype=torch.float16, device=dev)
            zero = torch.empty(H, 1, D, dtype=torch.float16, device=dev)
        else:
            scale = torch.empty(H, N, 1, dtype=torch.float16, device=dev)
            zero = torch.empty(H, N, 1, dtype=torch.float16, device=dev)
        out_data = torch.empty(H, N, n, dtype=torch.float16, device=dev) if n else None
        out_idx = torch.empty(n, dtype=torch.int16, device=dev) if n else None
        dest = dict_dest(codes, scale, zero, out_data, out_idx, N, D, bits, n, is_key)
        _C.quantize(x.data_ptr(), 0, N * D, D, None, 0, 1, H, N, D, bits, is_key, N, n, dest, None, dev)
        res = {"scale": scale, "zero": zero, "orig_dim": D, "bits": bits}
        if n:
            res["outlier_idx"] = out_idx.to(torch.int64)
            res["outlier_data"] = out_data
        res["codes"] = codes if self.packed else unpack(codes, bits, D)
        return res

    def _dequantize(self, q: dict, is_key: bool) -> torch.Tensor:
        codes = q["codes"]
        bits = q.get("bits", self.key_bits if is_key else self.value_bits)
        D = q["orig_dim"]
        if codes.shape[-1] != packed_width(D, bits):  # unpacked codes
            codes = pack(codes, bits)
        codes = codes.contiguous()
        H, N, _ = codes.shape
        n = int(q["outlier_idx"].numel()) if "outlier_idx" in q else 0
        scale = q["scale"].contiguous()
        zero = q["zero"].contiguous()
        od = q["outlier_data"].contiguous() if n else None
        oi = q["outlier_idx"].to(torch.int16).contiguous() if n else None
        src = dict_dest(codes, scale, zero, od, oi, N, D, bits, n, is_key)
        out = torch.empty(H, N, D, dtype=torch.float16, device=codes.device)
        rc = _C.load().akv_dequantize(ctypes.byref(src), None, 0, 0, 1, H, N, D, bits, int(is_key), n,
                                      out.data_ptr(), 0, N * D, D, None, _C.stream_of(codes))
        _C.check(rc, "akv_dequantize")
        return out

    # ------------------------------------------------------------------
    def quantize_keys(self, k: torch.Tensor) -> dict:
        """Per-channel quantisation of keys (H, N, D)."""
        return self._quantize(k, self.key_bits, True)

    def dequantize_keys(self, qk: dict) -> torch.Tensor:
        return self._dequantize(qk, True)

    def quantize_values(self, v: torch.Tensor) -> dict:
        """Per-token quantisation of values (H, N, D)."""
        return self._quantize(v, self.value_bits, False)

    def dequantize_values(self, qv: dict) -> torch.Tensor:
        return self._dequantize(qv, False)
