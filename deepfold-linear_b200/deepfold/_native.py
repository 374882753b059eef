"""Binding to ``libdfsink.so``, the C-ABI CUDA library behind every op here.

The library is built in-tree (``build_library``) with nvcc for sm_100a and
loaded with ctypes; the structures below mirror ``include/dfsink.h`` field by
field.  There is no fallback: if the library or a CUDA device is missing the
ops raise ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
import threading

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)                      # .../deepfold-linear_b200
CSRC_DIR = os.path.join(ROOT_DIR, "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(ROOT_DIR), "include")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libdfsink.so")
SOURCES = ["dfs_abi.cu", "dfs_fwd.cu", "dfs_bwd.cu", "dfs_stream.cu", "dfs_stream_bwd.cu", "dfs_stream_tma.cu",
           "dfs_stream_bwd_tma.cu", "dfs_selftest.cu", "dfs_noalloc.cu", "dfs_pad.cu", "dfs_dense.cu",
           "dfs_dense_grad.cu", "dfs_peer.cu"]
HEADERS = ["dfs_device.cuh", "dfs_kernels.cuh", "dfs_slab.cuh", "dfs_tma.cuh"]

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC"]
OBJ_DIR = os.path.join(LIB_DIR, "_obj")

# status codes (include/dfsink.h)
DFS_OK = 0
DFS_ERR_INVALID_ARGUMENT = 1
DFS_ERR_UNSUPPORTED = 2
DFS_ERR_WORKSPACE = 3
DFS_ERR_CUDA = 4
DFS_ERR_DEVICE_TIMEOUT = 8
DFS_ERR_NUMERIC = 16
DFS_WARN_CG_NOT_CONVERGED = 32

DFS_BF16, DFS_F16, DFS_F32 = 0, 1, 2
DFS_COST_QK, DFS_COST_DENSE = 0, 1

_P = ctypes.c_void_p


class DfsProblem(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("N", ctypes.c_int32),
                ("d", ctypes.c_int32), ("in_dtype", ctypes.c_int32), ("cost_mode", ctypes.c_int32),
                ("K_iter", ctypes.c_int32), ("check_every", ctypes.c_int32),
                ("lam", ctypes.c_float), ("r_0", ctypes.c_float), ("threshold", ctypes.c_float),
                ("cost_terms", ctypes.c_int32)]


DFS_TERM_POS, DFS_TERM_GEO, DFS_TERM_XRES = 1, 2, 4


class DfsFwdArgs(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "Q", "K", "V", "C", "x_res", "pos_weight", "pos_bins", "eps", "w_dist", "log_mu", "log_nu",
        "log_u_init", "log_v_init", "mask", "O", "x_centroid", "log_u", "log_v", "status", "T_norm",
        "r_head", "chain_id", "global_idx", "bond_matrix")]


class DfsCgParams(ctypes.Structure):
    _fields_ = [("rtol", ctypes.c_float), ("atol", ctypes.c_float), ("max_iter", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class DfsBwdArgs(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "Q", "K", "V", "x_res", "pos_weight", "pos_bins", "eps", "w_dist", "log_mu", "log_nu", "mask",
        "log_u", "log_v", "dO", "dxc", "dQ", "dK", "dV", "dlog_mu", "dlog_nu", "dx_res",
        "dpos_weight", "dw_dist", "cg_iters", "cg_residual", "status", "r_head", "dr_head",
        "chain_id", "global_idx", "bond_matrix")]


class DfsIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


DFS_MAX_PEERS = 8


class DfsPeerSet(ctypes.Structure):
    _fields_ = [("npeers", ctypes.c_int32), ("self", ctypes.c_int32),
                ("ws", ctypes.c_void_p * DFS_MAX_PEERS), ("wait_for", ctypes.c_uint64)]


EXPORTED_SYMBOLS = ("dfs_abi_version", "dfs_status_string", "dfs_max_n", "dfs_workspace_size",
                    "dfs_fwd", "dfs_bwd", "dfs_selftest_mma", "dfs_fwd_static", "dfs_stream_op",
                    "dfs_peer_alloc", "dfs_peer_open", "dfs_peer_close", "dfs_peer_free", "dfs_stream_op_peer",
                    "dfs_compute_bins", "dfs_peer_gather_rows", "dfs_stream_cg_loop_peer",
                    "dfs_dense_iterate", "dfs_dense_work_bytes", "dfs_dense_solve_bwd", "dfs_dense_solve_bwd_scratch",
                    "dfs_dense_transport_bwd")

# phases of the streamed path for row-sharded runs (include/dfsink.h)
DFS_OP_FWD_INIT, DFS_OP_FWD_ROWS, DFS_OP_FWD_COLS, DFS_OP_FWD_OUT = 0, 1, 2, 3
(DFS_OP_BWD_PREP, DFS_OP_BWD_ROWSTATS, DFS_OP_BWD_ROWDERIVE, DFS_OP_BWD_COLSTATS, DFS_OP_BWD_SETUP,
 DFS_OP_BWD_PT_T, DFS_OP_BWD_CGINIT, DFS_OP_BWD_P_U, DFS_OP_BWD_CGSTEP_FIRST, DFS_OP_BWD_CGSTEP,
 DFS_OP_BWD_P_X, DFS_OP_BWD_FINAL, DFS_OP_BWD_DQ, DFS_OP_BWD_DKV) = range(10, 24)
DFS_WS_FWD_F, DFS_WS_FWD_G = 0, 1
DFS_WS_BWD_M, DFS_WS_BWD_R, DFS_WS_BWD_D, DFS_WS_BWD_C, DFS_WS_BWD_GV, DFS_WS_BWD_T, DFS_WS_BWD_S = \
    2, 3, 4, 7, 8, 19, 20
DFS_WS_BWD_NSLOTS, DFS_WS_BWD_NSCALARS = 22, 8

# fixed device scratch behind dfs_fwd_static (DFS_STATIC_SCRATCH_BYTES in include/dfsink.h)
DFS_STATIC_SCRATCH_BYTES = 16 << 20

_lock = threading.RLock()  # ext() loads lib() while holding it
_lib = None


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC_DIR, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE_DIR, "dfsink.h")]
    return any(os.path.exists(f) and os.path.getmtime(f) > t for f in deps)


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libdfsink.so`` for sm_100a into the package (in-tree).

    Each source is compiled to an object file of its own (in parallel; only
    sources newer than their object, or any header, are recompiled), then the
    objects are linked into the shared library.
    """
    if not force and not _stale():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(OBJ_DIR, exist_ok=True)
    nvcc = os.environ.get("NVCC", "nvcc")
    hdr_time = max(os.path.getmtime(f) for f in [os.path.join(CSRC_DIR, h) for h in HEADERS]
                   + [os.path.join(INCLUDE_DIR, "dfsink.h")])

    def compile_one(src: str) -> str:
        s = os.path.join(CSRC_DIR, src)
        o = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        if not force and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_time):
            return o
        tmp_o = o + ".tmp.%d" % os.getpid()
        cmd = [nvcc] + NVCC_FLAGS + ["-I", INCLUDE_DIR, "-c", s, "-o", tmp_o]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(tmp_o, o)
        return o

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    tmp = LIB_PATH + ".tmp.%d" % os.getpid()
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp] + objs
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


TORCH_EXT_NAME = "dfsink_torch"
TORCH_EXT_PATH = os.path.join(LIB_DIR, TORCH_EXT_NAME + ".so")
TORCH_EXT_SOURCE = os.path.join(CSRC_DIR, "dfs_torch.cpp")
_ext = None


def build_torch_ext(force: bool = False, verbose: bool = False) -> str:
    """Compile the native autograd glue (``dfsink_torch.so``, linked to
    ``libdfsink.so``) into the package with torch's extension builder."""
    build_library(verbose=verbose)
    deps = [TORCH_EXT_SOURCE, LIB_PATH, os.path.join(INCLUDE_DIR, "dfsink.h")]
    if (not force and os.path.exists(TORCH_EXT_PATH)
            and all(os.path.getmtime(f) <= os.path.getmtime(TORCH_EXT_PATH) for f in deps)):
        return TORCH_EXT_PATH
    from torch.utils import cpp_extension

    bdir = os.path.join(LIB_DIR, "_build")
    os.makedirs(bdir, exist_ok=True)
    # the extension finds libdfsink.so beside itself ($ORIGIN, escaped for ninja ("$$") and
    # for the shell that runs the link ("\\$"))
    ldflags = [f"-L{LIB_DIR}", "-ldfsink", "-Wl,-rpath,\\$$ORIGIN:\\$$ORIGIN/.."]
    cpp_extension.load(name=TORCH_EXT_NAME, sources=[TORCH_EXT_SOURCE], extra_include_paths=[INCLUDE_DIR],
                       extra_cflags=["-O2"], extra_ldflags=ldflags, build_directory=bdir, with_cuda=True,
                       verbose=verbose, is_python_module=True)
    tmp = TORCH_EXT_PATH + ".tmp.%d" % os.getpid()
    with open(os.path.join(bdir, TORCH_EXT_NAME + ".so"), "rb") as src, open(tmp, "wb") as dst:
        dst.write(src.read())
    os.replace(tmp, TORCH_EXT_PATH)
    return TORCH_EXT_PATH


def ext():
    """The native autograd module (raises if it has not been built)."""
    global _ext
    if _ext is not None:
        return _ext
    with _lock:
        if _ext is None:
            if not os.path.exists(TORCH_EXT_PATH):
                raise RuntimeError(
                    f"{TORCH_EXT_NAME}.so not found at {TORCH_EXT_PATH}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'`")
            import importlib.util

            lib()  # libdfsink first (the extension links to it)
            spec = importlib.util.spec_from_file_location(TORCH_EXT_NAME, TORCH_EXT_PATH)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            _ext = mod
    return _ext


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libdfsink.so not found at {LIB_PATH}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` (needs nvcc)")
            L = ctypes.CDLL(LIB_PATH)
            L.dfs_abi_version.restype = ctypes.c_int
            L.dfs_status_string.restype = ctypes.c_char_p
            L.dfs_status_string.argtypes = [ctypes.c_int]
            L.dfs_max_n.restype = ctypes.c_int
            L.dfs_max_n.argtypes = [ctypes.c_int]
            L.dfs_workspace_size.restype = ctypes.c_int
            L.dfs_workspace_size.argtypes = [ctypes.POINTER(DfsProblem), ctypes.POINTER(ctypes.c_size_t),
                                             ctypes.POINTER(ctypes.c_size_t)]
            L.dfs_fwd.restype = ctypes.c_int
            L.dfs_fwd.argtypes = [ctypes.POINTER(DfsProblem), ctypes.POINTER(DfsFwdArgs), _P,
                                  ctypes.c_size_t, _P]
            L.dfs_bwd.restype = ctypes.c_int
            L.dfs_bwd.argtypes = [ctypes.POINTER(DfsProblem), ctypes.POINTER(DfsCgParams),
                                  ctypes.POINTER(DfsBwdArgs), _P, ctypes.c_size_t, _P]
            L.dfs_stream_op.restype = ctypes.c_int
            L.dfs_stream_op.argtypes = [ctypes.c_int, ctypes.POINTER(DfsProblem), ctypes.POINTER(DfsCgParams),
                                        ctypes.POINTER(DfsFwdArgs), ctypes.POINTER(DfsBwdArgs), ctypes.c_int,
                                        ctypes.c_int, _P, ctypes.c_size_t, _P]
            L.dfs_fwd_static.restype = ctypes.c_int
            L.dfs_fwd_static.argtypes = [ctypes.POINTER(DfsProblem), ctypes.POINTER(DfsFwdArgs), _P]
            L.dfs_peer_alloc.restype = ctypes.c_int
            L.dfs_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.POINTER(DfsIpcHandle)]
            L.dfs_peer_open.restype = ctypes.c_int
            L.dfs_peer_open.argtypes = [ctypes.POINTER(DfsIpcHandle), ctypes.POINTER(ctypes.c_void_p)]
            L.dfs_peer_close.restype = ctypes.c_int
            L.dfs_peer_close.argtypes = [_P]
            L.dfs_peer_free.restype = ctypes.c_int
            L.dfs_peer_free.argtypes = [_P]
            L.dfs_stream_op_peer.restype = ctypes.c_int
            L.dfs_stream_op_peer.argtypes = [ctypes.c_int, ctypes.POINTER(DfsProblem), ctypes.POINTER(DfsFwdArgs),
                                             ctypes.c_int, ctypes.c_int, _P, ctypes.c_size_t,
                                             ctypes.POINTER(DfsPeerSet), _P]
            L.dfs_peer_gather_rows.restype = ctypes.c_int
            L.dfs_peer_gather_rows.argtypes = [ctypes.POINTER(DfsPeerSet), ctypes.c_size_t, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_size_t, _P, _P]
            L.dfs_stream_cg_loop_peer.restype = ctypes.c_int
            L.dfs_stream_cg_loop_peer.argtypes = [ctypes.POINTER(DfsProblem), ctypes.POINTER(DfsCgParams),
                                                  ctypes.POINTER(DfsBwdArgs), ctypes.c_int, ctypes.c_int, _P,
                                                  ctypes.c_size_t, ctypes.POINTER(DfsPeerSet), ctypes.c_size_t, _P]
            _I, _F = ctypes.c_int, ctypes.c_float
            L.dfs_dense_iterate.restype = ctypes.c_int
            L.dfs_dense_iterate.argtypes = [_I, _I, _I, _F] + [_P] * 8 + [_I, _I] + [_P] * 6
            L.dfs_dense_work_bytes.restype = ctypes.c_size_t
            L.dfs_dense_work_bytes.argtypes = [_I, _I, _I]
            L.dfs_dense_solve_bwd_scratch.restype = ctypes.c_size_t
            L.dfs_dense_solve_bwd_scratch.argtypes = [_I, _I, _I, _I]
            L.dfs_dense_solve_bwd.restype = ctypes.c_int
            L.dfs_dense_solve_bwd.argtypes = [_I, _I, _I, _I, _F] + [_P] * 15
            L.dfs_dense_transport_bwd.restype = ctypes.c_int
            L.dfs_dense_transport_bwd.argtypes = [_I, _I, _I] + [_P] * 5
            L.dfs_compute_bins.restype = ctypes.c_int
            L.dfs_compute_bins.argtypes = [ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _P]
            L.dfs_selftest_mma.restype = ctypes.c_int
            L.dfs_selftest_mma.argtypes = [ctypes.c_int, _P, _P, _P, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, _P]
            _lib = L
    return _lib


def status_string(code: int) -> str:
    return lib().dfs_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != DFS_OK:
        raise RuntimeError(f"{what} failed: {status_string(code)} (code {code})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return DFS_BF16
    if dt == torch.float16:
        return DFS_F16
    if dt == torch.float32:
        return DFS_F32
    raise TypeError(f"unsupported dtype {dt}; expected bfloat16, float16 or float32")


def make_problem(B, H, N, d, dtype, K_iter, lam, r_0, cost_mode=DFS_COST_QK, threshold=None,
                 check_every=2, cost_terms=0) -> DfsProblem:
    return DfsProblem(B=B, H=H, N=N, d=d, in_dtype=dtype_code(dtype), cost_mode=cost_mode,
                      K_iter=int(K_iter), check_every=int(check_every),
                      lam=float(lam) if not math.isinf(lam) else float("inf"), r_0=float(r_0),
                      threshold=float(threshold) if threshold is not None else 0.0,
                      cost_terms=int(cost_terms))


def workspace_bytes(prob: DfsProblem) -> tuple[int, int]:
    """(forward, backward) workspace bytes of a problem (dfs_workspace_size)."""
    fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    check(lib().dfs_workspace_size(prob, ctypes.byref(fb), ctypes.byref(bb)), "dfs_workspace_size")
    return fb.value, bb.value


def max_n(d: int) -> int:
    return int(lib().dfs_max_n(int(d)))


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("deepfold B200 Sinkhorn ops run on CUDA tensors only (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("all tensors must be on the same CUDA device")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev
