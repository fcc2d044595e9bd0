"""Binding to the C ABI in ``include/insitu_b200.h`` (``libinsitu_b200.so``).

The shared library is built in-tree by :func:`build` (nvcc, sm_100a). Loading
never falls back to anything: a missing or unloadable library raises, because
a silent CPU path would make every GPU parity claim meaningless.
"""

from __future__ import annotations

import ctypes as C
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libinsitu_b200.so")
SOURCES = ("csrc/insitu.cu", "csrc/common.cuh", "csrc/kernels.cuh", "csrc/scan_chunked.cuh",
           "csrc/scan_fused.cuh", "csrc/project.cuh")
HEADER = os.path.join(ROOT, "include", "insitu_b200.h")

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared", "-Xlinker", "-soname=libinsitu_b200.so"]

# status codes (insitu_b200.h)
INS_OK, INS_EBADLEN, INS_ETIMEOUT, INS_ERANGE, INS_EINVAL, INS_ENOMEM, INS_ECUDA = 0, 4, 5, 7, 8, 9, 10
INS_SOFTMAX_ONLINE, INS_SOFTMAX_TWO_PASS = 0, 1
INS_INGRESS_PREROTATED = 1
INS_TILES = {"auto": 0, "large": 1, "small": 2}
INS_SCAN = {"fused": 0, "split": 1}


class InsituError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[status {code}] {msg}")
        self.code = code


class CapacityError(InsituError, ValueError):
    """The reference raises ValueError when a cache is full (cache/base.py:67-73)."""


class ArgumentError(InsituError, ValueError):
    pass


class RangeError(InsituError, OverflowError):
    """A value escaped its fixed-point format (the board's ATTN_ERANGE)."""


class DeviceTimeout(InsituError, TimeoutError):
    """A bounded device-side wait gave up (the board's ATTN_ETIMEOUT)."""


_ERRORS = {INS_EBADLEN: CapacityError, INS_EINVAL: ArgumentError, INS_ERANGE: RangeError,
           INS_ETIMEOUT: DeviceTimeout}


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "head_dim", "n_kv_heads", "kv_groups", "key_bits", "value_bits", "norm_bits", "norm_frac",
        "qk_frac", "centroid_frac", "acc_frac", "acc_width", "score_width", "prob_frac",
        "exp_lut_bits", "saturate", "rot_rounds", "rot_shift", "rot_inv_sqrt_q15", "page_tokens",
        "max_seqs", "max_pages_per_seq", "reserved0")] + [("n_pages", C.c_int64)]


class Tables(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_int64)) for n in (
        "signs", "k_centroids", "k_bounds", "v_centroids", "v_bounds", "exp_table")] + [
        ("log2e", C.c_int64), ("delta_max", C.c_int64)]


class Stats(C.Structure):
    """AttentionStats (ops/attention.py:257-274)."""
    _fields_ = [(n, C.c_int64) for n in (
        "n_tokens", "rescale_events", "score_overflows", "acc_overflows", "max_abs_score",
        "max_abs_acc")]


STATS_FIELDS = tuple(n for n, _ in Stats._fields_)


class SeamCfg(C.Structure):
    """ins_seam_cfg."""
    _fields_ = [("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("norm_eps", C.c_float),
                ("cast_after_rope", C.c_int32), ("attn_scale", C.c_double),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("rope_frac", C.c_int32),
                ("max_position", C.c_int32)]

# every symbol the header declares, for the load check
SYMBOLS = ("ins_abi_version", "ins_bytes_per_token", "ins_cache_create", "ins_cache_destroy",
           "ins_cache_reset", "ins_cache_length", "ins_cache_capacity", "ins_ingress", "ins_rotate",
           "ins_scores", "ins_scan", "ins_cache_export", "ins_cache_import", "ins_cache_status",
           "ins_last_error", "ins_scan_noalloc", "ins_scan_recomputed", "ins_part_bytes",
           "ins_scan_maxima", "ins_scan_part", "ins_merge_parts", "ins_cache_set_tiles",
           "ins_ingress_lanes", "ins_lanes_bytes_per_token", "ins_ddr_image_bytes",
           "ins_cache_ddr_image", "ins_seam", "ins_seam_device_positions",
           "ins_cache_launches", "ins_finalize", "ins_exp_lut",
           "ins_scan_recomputed_total", "ins_cache_set_scan_kernel", "ins_cache_set_wait_test",
           "ins_project")


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build insitu_b200")


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libinsitu_b200.so`` in-tree for sm_100a."""
    srcs = [os.path.join(HERE, s) for s in SOURCES] + [HEADER]
    if not force and os.path.exists(LIB_PATH):
        newest = max(os.path.getmtime(s) for s in srcs)
        if os.path.getmtime(LIB_PATH) >= newest:
            return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, os.path.join(HERE, "csrc", "insitu.cu")]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=HERE)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


TORCH_OPS_PATH = os.path.join(HERE, "libinsitu_torch.so")
TORCH_OPS_SOURCE = os.path.join(HERE, "csrc", "torch_ops.cpp")


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Compile the thin torch extension (``csrc/torch_ops.cpp``) in-tree,
    linked against ``libinsitu_b200.so`` (found next to it at run time)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension
    srcs = [TORCH_OPS_SOURCE, HEADER]
    if not force and os.path.exists(TORCH_OPS_PATH):
        if os.path.getmtime(TORCH_OPS_PATH) >= max(os.path.getmtime(s) for s in srcs):
            return TORCH_OPS_PATH
    build(verbose=verbose)
    inc = [f"-I{p}" for p in cpp_extension.include_paths(device_type="cuda")]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths(device_type="cuda")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_OPS_PATH + ".tmp"
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *inc, f"-I{sysconfig.get_paths()['include']}",
           TORCH_OPS_SOURCE, "-o", tmp, *libdirs, f"-L{HERE}", "-linsitu_b200",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=HERE)
    os.replace(tmp, TORCH_OPS_PATH)
    return TORCH_OPS_PATH


_ops = None


def ops():
    """The torch operators of the extension (torch.ops.insitu). Raises if the
    extension was never built -- there is no fallback."""
    global _ops
    if _ops is not None:
        return _ops
    import torch
    lib()                                   # the C ABI first, so the extension resolves against it
    if not os.path.exists(TORCH_OPS_PATH):
        raise RuntimeError(f"{TORCH_OPS_PATH} is missing: build it with "
                           "insitu_b200._lib.build_torch_ops(). insitu_b200 has no fallback.")
    torch.ops.load_library(TORCH_OPS_PATH)
    _ops = torch.ops.insitu
    return _ops


_lib = None


def lib():
    """The loaded library. Raises if it was never built -- there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with insitu_b200._lib.build() (nvcc, sm_100a). "
            "insitu_b200 has no CPU fallback.")
    L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)   # the torch extension binds to this copy
    vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
    L.ins_abi_version.restype = i32
    L.ins_bytes_per_token.argtypes = [C.POINTER(Config)]
    L.ins_bytes_per_token.restype = i32
    L.ins_cache_create.argtypes = [C.POINTER(Config), C.POINTER(Tables), i32, C.POINTER(vp)]
    L.ins_cache_destroy.argtypes = [vp]
    L.ins_cache_reset.argtypes = [vp, i32]
    L.ins_cache_length.argtypes = [vp, i32]
    L.ins_cache_length.restype = i64
    L.ins_cache_capacity.argtypes = [vp]
    L.ins_cache_capacity.restype = i64
    L.ins_ingress.argtypes = [vp, i32, vp, vp, vp, vp, vp, C.c_uint32, vp]
    L.ins_rotate.argtypes = [vp, i64, vp, vp, vp]
    L.ins_scores.argtypes = [vp, i32, i32, i64, i64, vp, vp, vp, vp]
    L.ins_scan.argtypes = [vp, i32, vp, vp, vp, vp, vp, C.c_int, vp]
    L.ins_scan_noalloc.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    L.ins_cache_export.argtypes = [vp, i32, i32, i64, i64, vp]
    L.ins_cache_import.argtypes = [vp, i32, i64, vp]
    L.ins_cache_status.argtypes = [vp, vp]
    L.ins_scan_recomputed.argtypes = [vp, vp]
    L.ins_scan_recomputed.restype = i64
    L.ins_scan_recomputed_total.argtypes = [vp, vp]
    L.ins_scan_recomputed_total.restype = i64
    L.ins_part_bytes.argtypes = [vp, i32]
    L.ins_part_bytes.restype = i64
    L.ins_scan_maxima.argtypes = [vp, i32, vp, vp, vp, vp, vp]
    L.ins_scan_part.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    L.ins_merge_parts.argtypes = [vp, i32, i32, vp, vp, vp, vp]
    L.ins_cache_set_tiles.argtypes = [vp, i32]
    L.ins_cache_set_scan_kernel.argtypes = [vp, i32]
    L.ins_cache_set_wait_test.argtypes = [vp, i32, i32, i32, i32]
    L.ins_ingress_lanes.argtypes = [vp, i32, vp, vp, vp, vp]
    L.ins_lanes_bytes_per_token.argtypes = [vp]
    L.ins_lanes_bytes_per_token.restype = i64
    L.ins_ddr_image_bytes.argtypes = [vp, i64]
    L.ins_ddr_image_bytes.restype = i64
    L.ins_cache_ddr_image.argtypes = [vp, i32, i64, vp, vp]
    L.ins_seam.argtypes = [vp, i32, vp, vp, vp, vp, C.POINTER(SeamCfg), vp, vp, vp, vp, vp]
    L.ins_seam_device_positions.argtypes = L.ins_seam.argtypes
    L.ins_finalize.argtypes = [vp, i64, vp, vp, vp, vp, vp, vp]
    L.ins_exp_lut.argtypes = [vp, i64, vp, vp, vp]
    L.ins_project.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp]
    L.ins_cache_launches.argtypes = [vp]
    L.ins_cache_launches.restype = i64
    L.ins_last_error.restype = C.c_char_p
    _lib = L
    return L


def check(rc: int) -> None:
    if rc == INS_OK:
        return
    msg = lib().ins_last_error().decode(errors="replace")
    raise _ERRORS.get(rc, InsituError)(rc, msg)
