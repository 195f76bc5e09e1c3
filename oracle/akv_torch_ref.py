"""Torch CPU restatement of the reference's decode path.  TEST / BENCHMARK INFRASTRUCTURE ONLY.

The timed CPU arm of ``bench.py`` (``--impl reference`` and ``cpu_baseline``)
runs the reference's own CPU recipe for one mixed-tier decode step with torch's
CPU kernels on every host core (``torch.set_num_threads``), as the reference
does when it runs on a CPU tensor:

* ``bitpack.unpack`` (akv/bitpack.py:22-30, :54-68, :82-90) of the packed codes;
* ``AffineQuantizer.dequantize_keys/values`` (akv/affine_quantizer.py:112-124,
  :178-189): ``codes.half() * scale + zero`` in fp16, outlier channels
  overwritten with their fp16 originals;
* ``mixed_precision_decode_attention`` (akv/fused_attention.py:324-366):
  ``torch.cat`` of the two tiers, fp32 ``matmul`` with the query, ``softmax``,
  fp32 ``matmul`` with the values.

The reference dequantises one quantiser call at a time; here the calls of a
(row, KV head) unit are batched into one tensor op per step (same arithmetic,
fewer Python round trips), so the timed CPU path is, if anything, faster than
the reference's.  The packed inputs come from the numpy oracle
(``oracle.akv_oracle``), outside the timed region.  Nothing in the product
package imports this module.
"""
from __future__ import annotations

import math
import time

import numpy as np
import torch


def unpack(packed: torch.Tensor, bits: int, dim: int) -> torch.Tensor:
    """uint8 (..., dim*bits/8) -> uint8 codes (..., dim), the reference's byte layouts."""
    p = packed.to(torch.int32)
    if bits == 4:  # even index in the high nibble
        out = torch.stack([(p >> 4) & 15, p & 15], -1)
    elif bits == 2:  # four codes per byte, MSB first
        out = torch.stack([(p >> 6) & 3, (p >> 4) & 3, (p >> 2) & 3, p & 3], -1)
    else:  # 8 codes in a 24-bit big-endian word
        g = p.reshape(*p.shape[:-1], -1, 3)
        w = (g[..., 0] << 16) | (g[..., 1] << 8) | g[..., 2]
        out = torch.stack([(w >> (21 - 3 * j)) & 7 for j in range(8)], -1)
    return out.reshape(*packed.shape[:-1], -1)[..., :dim].to(torch.uint8)


def stack_groups(groups: list, bits: int, is_key: bool) -> dict:
    """Oracle quantiser dicts of one (row, KV head) unit (one per 32-token
    group, H = 1) -> batched torch tensors: codes (G, 32, packed), scale /
    zero (G, 1, D) for keys or (G, 32, 1) for values, outlier ids (G, n) and
    originals (G, 32, n)."""
    codes = torch.from_numpy(np.stack([g["codes"][0] for g in groups]))
    scale = torch.from_numpy(np.stack([g["scale"][0] for g in groups]))
    zero = torch.from_numpy(np.stack([g["zero"][0] for g in groups]))
    res = {"codes": codes, "scale": scale, "zero": zero, "bits": bits, "dim": groups[0]["orig_dim"]}
    if "outlier_idx" in groups[0]:
        res["outlier_idx"] = torch.from_numpy(np.stack([g["outlier_idx"] for g in groups]))
        res["outlier_data"] = torch.from_numpy(np.stack([g["outlier_data"][0] for g in groups]))
    return res


def dequantize(q: dict) -> torch.Tensor:
    """akv/affine_quantizer.py:112-124 / :178-189 over stacked groups: fp16 (G*32, D)."""
    out = unpack(q["codes"], q["bits"], q["dim"]).to(torch.float16) * q["scale"] + q["zero"]
    if "outlier_idx" in q:
        idx = q["outlier_idx"]  # (G, n): channel ids of each group
        out.scatter_(2, idx[:, None, :].expand(-1, out.shape[1], -1), q["outlier_data"])
    return out.reshape(-1, out.shape[-1])


def decode_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    """akv/fused_attention.py:362-366 for one KV head: q (g, D) fp16, keys/values (N, D) fp16 -> fp32 (g, D)."""
    sm_scale = 1.0 / math.sqrt(q.shape[-1])
    qk = torch.matmul(q.float(), keys.float().transpose(-2, -1)) * sm_scale
    attn = torch.softmax(qk, dim=-1)
    return torch.matmul(attn, values.float())


def unit_inputs(seed: int, n_warm: int, n_hot: int, D: int, g: int, key_bits: int, value_bits: int,
                outlier_fraction: float) -> tuple:
    """Seeded inputs of one (row, KV head) unit: the warm tier quantised by the
    numpy oracle in 32-token groups, the FP16 hot window and g query heads."""
    from oracle import akv_oracle as O
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((1, 1, n_warm, D)).astype(np.float16)
    v = rng.standard_normal((1, 1, n_warm, D)).astype(np.float16)
    gk = O.quantize_groups(k, key_bits, 32, True, outlier_fraction)[0]
    gv = O.quantize_groups(v, value_bits, 32, False, outlier_fraction)[0]
    hk = torch.from_numpy(rng.standard_normal((n_hot, D)).astype(np.float16))
    hv = torch.from_numpy(rng.standard_normal((n_hot, D)).astype(np.float16))
    q = torch.from_numpy(rng.standard_normal((g, D)).astype(np.float16))
    return stack_groups(gk, key_bits, True), stack_groups(gv, value_bits, False), hk, hv, q


def decode_unit(wk: dict, wv: dict, hk: torch.Tensor, hv: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """One unit of the reference's CPU decode step: dequantise the warm tier, concatenate, attend."""
    keys = torch.cat([hk, dequantize(wk)], 0)
    values = torch.cat([hv, dequantize(wv)], 0)
    return decode_attention(q, keys, values)


def time_units(seeds, threads: int, **shape) -> float:
    """Mean seconds of decode_unit over the given seeds with torch on `threads`
    CPU threads (inputs built outside the timed region)."""
    torch.set_num_threads(threads)
    ts = []
    for s in seeds:
        args = unit_inputs(s, **shape)
        decode_unit(*args)  # first touch of the buffers
        t = time.perf_counter()
        decode_unit(*args)
        ts.append(time.perf_counter() - t)
    return float(np.mean(ts))


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"
