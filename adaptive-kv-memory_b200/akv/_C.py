"""ctypes binding of libakv_sm100.so (the C ABI in include/akv_b200.h).

The library is built in-tree by ``adaptive-kv-memory_b200/build.py`` into
``akv/_lib/libakv_sm100.so``.  There is no fallback: if the library is
missing, every warm-tier op raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p, c_char_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libakv_sm100.so")

AKV_OK = 0
AKV_ERR_WORKSPACE = -8
BLOCK_TOKENS = 32
ERRORS = {
    -1: "AKV_ERR_SHAPE", -2: "AKV_ERR_BITS", -3: "AKV_ERR_ALIGN", -4: "AKV_ERR_UNSUPPORTED",
    -5: "AKV_ERR_LAUNCH", -6: "AKV_ERR_TIMEOUT", -7: "AKV_ERR_NULL", -8: "AKV_ERR_WORKSPACE",
}


class View(ctypes.Structure):
    """akv_view: addr(b, h, blk, slot) = ptr + b*sb + h*sh + blk*sblk + slot*sslot (bytes)."""
    _fields_ = [("ptr", c_void_p), ("sb", c_int64), ("sh", c_int64), ("sblk", c_int64), ("sslot", c_int64)]


class QDest(ctypes.Structure):
    """akv_qdest: where one quantiser call writes (or one dequantiser call reads)."""
    _fields_ = [(n, View) for n in ("codes", "scale", "zero", "out_data", "out_idx", "out_vdq", "mask", "flags")] + \
        [("pair_order", c_int32)]



class WarmLayout(ctypes.Structure):
    """akv_warm_layout: byte offsets inside one 32-token warm block record."""
    _fields_ = [(n, c_int32) for n in ("head_dim", "key_bits", "value_bits", "n_outlier", "kc", "vc", "ks",
                                        "kz", "vs", "vz", "ko", "vo", "vd", "ki", "vi", "mask", "flags",
                                        "bytes")]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}

class DecodeArgs(ctypes.Structure):
    """akv_decode_args (include/akv_b200.h)."""
    _fields_ = [("q", c_void_p), ("q_sb", c_int64), ("q_sh", c_int64), ("hot_k", c_void_p), ("hot_v", c_void_p),
                ("h_sb", c_int64), ("h_sh", c_int64), ("h_sn", c_int64), ("n_hot", c_int32), ("hot_len", c_void_p),
                ("warm", c_void_p), ("w_sb", c_int64), ("w_sh", c_int64), ("layout", c_void_p),
                ("n_warm_blocks", c_int32), ("warm_len", c_void_p), ("B", c_int32), ("Hq", c_int32),
                ("Hkv", c_int32), ("D", c_int32), ("sm_scale", c_float), ("out", c_void_p), ("o_sb", c_int64),
                ("o_sh", c_int64), ("lse", c_void_p), ("partial_out", c_void_p), ("workspace", c_void_p),
                ("workspace_bytes", c_size_t), ("workspace_need", c_void_p), ("status", c_void_p)]


class LayerStep(ctypes.Structure):
    """akv_layer_step (include/akv_b200.h): one AKVLayer's steady decode-step state."""
    _fields_ = [("hot_k", c_void_p), ("hot_v", c_void_p), ("h_sb", c_int64), ("h_sh", c_int64), ("h_sn", c_int64),
                ("hot_rows", c_int64), ("arena", c_void_p), ("a_sb", c_int64), ("a_sh", c_int64),
                ("layout", WarmLayout), ("B", c_int32), ("H", c_int32), ("n_blocks", c_int32),
                ("max_blocks", c_int32), ("phys", c_void_p), ("hpos", c_void_p), ("imp", c_void_p),
                ("lo", c_int64), ("hi", c_int64), ("cap", c_int64), ("wslots", c_void_p), ("wpos", c_void_p),
                ("slot_pos", c_void_p), ("n_wslots", c_int64), ("cap_wslots", c_int64), ("n_wpos", c_int64),
                ("cap_wpos", c_int64), ("cap_slot_pos", c_int64), ("protect_first", c_int32),
                ("protect_recent", c_int32), ("decay", c_float), ("total_len", c_int64), ("step", c_int64),
                ("warm_len", c_int64), ("warm_bytes_packed", c_int64), ("bytes_per_event", c_int64),
                ("status", c_void_p)]


# name -> (restype, argtypes); must list every function declared in akv_b200.h
SIGNATURES = {
    "akv_strerror": (c_char_p, [c_int]),
    "akv_abi_version": (c_int, []),
    "akv_warm_layout_init": (c_int, [c_int, c_int, c_int, c_int, POINTER(WarmLayout)]),
    "akv_pack_codes": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "akv_unpack_codes": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "akv_quantize": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                             c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                             POINTER(QDest), c_void_p, c_void_p]),
    "akv_quantize_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "akv_quantize_ws": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                POINTER(QDest), c_void_p, c_size_t, c_void_p, c_void_p]),
    "akv_outlier_norm_sums_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "akv_outlier_norm_sums": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                      c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p,
                                      c_void_p]),
    "akv_quantize_ext": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                 c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                 POINTER(QDest), c_void_p, c_int, c_void_p, c_size_t, c_void_p, c_void_p]),
    "akv_dequantize": (c_int, [POINTER(QDest), c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int,
                               c_int, c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "akv_warm_append_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "akv_warm_append": (c_int, [c_void_p, c_int64, c_int64, POINTER(WarmLayout), c_int, c_void_p, c_int64, c_int64,
                                c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int,
                                c_int, c_int, c_int, c_void_p, c_size_t, c_void_p, c_void_p]),
    "akv_warm_demote_install": (c_int, [c_void_p, c_int64, c_int64, POINTER(WarmLayout), c_int, c_void_p, c_int64,
                                        c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
                                        c_int64, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "akv_mixed_decode_args": (c_int, [POINTER(DecodeArgs), c_void_p]),
    "akv_layer_decode_step": (c_int, [POINTER(LayerStep), c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                      c_void_p]),
    "akv_peer_alloc": (c_int, [c_size_t, c_void_p]),
    "akv_peer_free": (c_int, [c_void_p]),
    "akv_ipc_export": (c_int, [c_void_p, c_void_p]),
    "akv_ipc_open": (c_int, [c_void_p, c_void_p]),
    "akv_ipc_close": (c_int, [c_void_p]),
    "akv_peer_publish": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                                 c_void_p]),
    "akv_peer_combine": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_void_p,
                                 c_void_p, c_void_p]),
    "akv_int4_group_dequant": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                       c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p]),
    "akv_group_dequant": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                  c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "akv_group_quantize": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p,
                                   c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "akv_attention_probs": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64,
                                    c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_int64,
                                    c_int64, c_int64, c_int, c_void_p]),
    "akv_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "akv_mixed_decode": (c_int, [c_void_p, c_int64, c_int64,
                                 c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p,
                                 c_void_p, c_int64, c_int64, POINTER(WarmLayout), c_int, c_void_p,
                                 c_int, c_int, c_int, c_int, c_float,
                                 c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                 c_void_p, c_size_t, c_void_p, c_void_p]),
    "akv_mixed_decode_paged": (c_int, [c_void_p, c_int64, c_int64,
                                       c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p,
                                       c_void_p, c_int, c_int64, c_int64, c_void_p, c_int64, POINTER(WarmLayout),
                                       c_int, c_void_p,
                                       c_int, c_int, c_int, c_int, c_float,
                                       c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                       c_void_p, c_size_t, c_void_p, c_void_p]),
    "akv_mixed_decode_noalloc": (c_int, [c_void_p, c_int64, c_int64,
                                         c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p,
                                         c_void_p, c_int64, c_int64, POINTER(WarmLayout), c_int, c_void_p,
                                         c_int, c_int, c_int, c_int, c_float,
                                         c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                         c_void_p, c_void_p]),
    "akv_prefill_attention": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int,
                                      c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p, c_int64,
                                      c_void_p, c_int64, c_int64, POINTER(WarmLayout), c_int, c_void_p, c_int64,
                                      c_int, c_int, c_int, c_int, c_float,
                                      c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "akv_lse_combine": (c_int, [c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_void_p, c_int64, c_void_p,
                                c_void_p, c_void_p]),
    "akv_set_reduction_width": (c_int, [c_int]),
    "akv_importance_update": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_float, c_void_p]),
    "akv_migrator_update": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                                    c_int64, c_float, c_void_p]),
    "akv_migrator_importance": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_float, c_float, c_float,
                                        c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "akv_select_workspace_bytes": (c_size_t, [c_int]),
    "akv_select_bottomk": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "akv_gather_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int, c_int, c_int,
                                c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "akv_scatter_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int,
                                 c_int, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "akv_selftest_wait": (c_int, [c_int, c_int64, c_void_p, c_void_p, c_void_p]),
    "akv_cold_copy": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p]),
}

_lib = None


def lib_path() -> str:
    return LIB_PATH


def load():
    """Load the library (once) and bind every ABI symbol.  Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"akv: native library not found at {LIB_PATH}; build it with "
            "`python adaptive-kv-memory_b200/build.py` (no CPU fallback exists)")
    import torch  # noqa: F401  (makes torch's libcudart visible to the loader first)
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    lib.akv_set_reduction_width(cpu_reduction_width())
    _lib = lib
    return lib


def cpu_reduction_width() -> int:
    """Floats per SIMD register torch's CPU kernels use on this host (16 with
    AVX-512, 8 otherwise): the importance sums follow the reference's torch
    CPU reduction order on the same machine."""
    import torch
    try:
        cap = torch.backends.cpu.get_cpu_capability()
    except Exception:
        cap = ""
    return 16 if "AVX512" in str(cap).upper() else 8


def strerror(rc: int) -> str:
    return load().akv_strerror(rc).decode()


def check(rc: int, what: str) -> None:
    if rc != AKV_OK:
        raise RuntimeError(f"{what} failed: {ERRORS.get(rc, rc)} ({strerror(rc)})")


def ptr(t) -> int | None:
    """Device/host address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


_raw_stream = None


def stream_of(t) -> int:
    """The current torch stream handle for the tensor's device (as an int).

    Called on every op of the hot path, so it asks torch's raw-stream accessor
    (a few hundred ns) rather than building a Stream object (~10 us)."""
    global _raw_stream
    import torch
    if _raw_stream is None:
        _raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", False)
    if _raw_stream:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("akv: warm-tier ops run on CUDA tensors only (no CPU fallback)")


def warm_layout(head_dim: int, key_bits: int, value_bits: int, n_outlier: int) -> WarmLayout:
    L = WarmLayout()
    check(load().akv_warm_layout_init(head_dim, key_bits, value_bits, n_outlier, ctypes.byref(L)),
          "akv_warm_layout_init")
    return L


_ws_sizes: dict = {}


def workspace_bytes(name: str, *args) -> int:
    """Memoised workspace-size query (``akv_*_workspace_bytes``): pure
    functions of their shape arguments, asked on every call of the hot path."""
    key = (name,) + args
    n = _ws_sizes.get(key)
    if n is None:
        n = _ws_sizes[key] = int(getattr(load(), name)(*args))
    return n


def quantize(x_ptr: int, sb: int, sh: int, sn: int, tok_ptr, tok_sb: int, B: int, H: int, N: int, D: int,
             bits: int, is_key: bool, group: int, n_out: int, dest: QDest, status_ptr, device,
             score_sum=None, score_heads: int = 0, n_src: int = 0) -> None:
    """akv_quantize_ext with a workspace from torch's allocator when the shape needs one
    (``score_sum``: all-reduced outlier norm sums when heads are sharded over GPUs; ``n_src``:
    rows the source holds, the bound the kernel checks each ``tok_ptr`` index against)."""
    import torch
    lib = load()
    need = workspace_bytes("akv_quantize_workspace_bytes", B, H, N, D, group, n_out, int(is_key))
    ws = torch.empty(need + 256, dtype=torch.uint8, device=device) if need else None
    wp = None if ws is None else (ws.data_ptr() + 255) // 256 * 256
    if tok_ptr is not None and n_src <= 0:
        raise ValueError("akv_quantize: a token index list needs the source row count n_src")
    rc = lib.akv_quantize_ext(x_ptr, sb, sh, sn, tok_ptr, tok_sb, n_src, B, H, N, D, bits, int(is_key), group, n_out,
                              ctypes.byref(dest), None if score_sum is None else score_sum.data_ptr(), score_heads,
                              wp, need, status_ptr, _stream_of_device(device))
    check(rc, "akv_quantize")


def _stream_of_device(device) -> int:
    import torch
    d = torch.device(device)
    global _raw_stream
    if _raw_stream is None:
        _raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", False)
    if _raw_stream:
        return _raw_stream(d.index if d.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(d).cuda_stream


def outlier_norm_sums(x, tok_idx, N: int, group: int, status=None):
    """(B, n_groups, D) fp32: per scale group, the sum over x's heads of the per-(head, channel) L2 norms."""
    import torch
    lib = load()
    B, H, _, D = x.shape
    n_groups = (N + group - 1) // group
    out = torch.empty(B, n_groups, D, dtype=torch.float32, device=x.device)
    need = lib.akv_outlier_norm_sums_workspace_bytes(B, H, N, D, group)
    ws = torch.empty(need + 256, dtype=torch.uint8, device=x.device)
    wp = (ws.data_ptr() + 255) // 256 * 256
    ti = None if tok_idx is None else tok_idx.contiguous()
    rc = lib.akv_outlier_norm_sums(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
                                   None if ti is None else ti.data_ptr(), 0 if ti is None or ti.dim() == 1 else ti.stride(0),
                                   x.shape[2], B, H, N, D, group, out.data_ptr(), wp, need,
                                   None if status is None else status.data_ptr(),
                                   torch.cuda.current_stream(x.device).cuda_stream)
    check(rc, "akv_outlier_norm_sums")
    return out
