"""C-ABI checks that need no GPU: the library loads, exports every entry point
declared in include/dfsink.h, and rejects bad arguments on the host before any
CUDA call is made."""

import ctypes
import os
import re

import pytest

from deepfold import _native as nat

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "dfsink.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(dfs_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    nat.build_library()
    return nat.lib()


def test_header_declares_the_expected_entry_points():
    assert set(declared_functions()) == set(nat.EXPORTED_SYMBOLS)


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_strings(lib):
    assert lib.dfs_abi_version() == 2
    assert nat.status_string(nat.DFS_OK) == "ok"
    assert "workspace" in nat.status_string(nat.DFS_ERR_WORKSPACE)
    assert nat.max_n(32) >= 384
    # head dims up to 64 run (others zero-padded to 32 or 64); beyond 64 nothing
    assert nat.max_n(8) == nat.max_n(48) == nat.max_n(64) == 1 << 16
    assert nat.max_n(96) == 0 and nat.max_n(0) == 0


def test_struct_sizes_match_header_layout():
    # every pointer field is 8 bytes; the problem block is 8 int32 + 4 floats
    assert ctypes.sizeof(nat.DfsProblem) == 48
    assert ctypes.sizeof(nat.DfsFwdArgs) == 24 * 8
    assert ctypes.sizeof(nat.DfsBwdArgs) == 31 * 8
    assert ctypes.sizeof(nat.DfsCgParams) == 16


def test_host_side_validation(lib):
    p = nat.make_problem(2, 8, 384, 32, __import__("torch").bfloat16, 20, float("inf"), 10.0)
    a = nat.DfsFwdArgs()
    assert lib.dfs_fwd(p, a, None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    fake = nat.DfsFwdArgs(Q=16, K=16, V=16, eps=16, log_mu=16, log_nu=16, log_u=16, log_v=16)
    # beyond the resident range the streamed kernels need a workspace
    big = nat.make_problem(1, 1, 4096, 32, __import__("torch").bfloat16, 20, 1.0, 10.0)
    assert lib.dfs_fwd(big, fake, None, 0, None) == nat.DFS_ERR_WORKSPACE
    fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.dfs_workspace_size(big, ctypes.byref(fb), ctypes.byref(bb)) == nat.DFS_OK
    # f, g, m, R (fp32, N each), fp32 copies of Q, K and V^T (N x d each), column-split
    # partials (3 x 128 fp32 for each CTA of up to 8 splits per 128-row block) and counters (one per
    # 128-row block), alignment slack, the peer-exchange arrival counter's slot and one (lo, hi)
    # valid extent per batch element
    splits = 8 * (4096 // 128) * 3 * 128 * 4
    assert fb.value == 4 * 4 * 4096 + 3 * 4 * 4096 * 32 + splits + 4 * (4096 // 128) + 2 * 256 + 128 + 8
    huge = nat.make_problem(1, 1, 1 << 17, 32, __import__("torch").bfloat16, 20, 1.0, 10.0)
    assert lib.dfs_fwd(huge, fake, None, 0, None) == nat.DFS_ERR_UNSUPPORTED
    wide_d = nat.make_problem(1, 1, 128, 96, __import__("torch").bfloat16, 20, 1.0, 10.0)
    assert lib.dfs_fwd(wide_d, fake, None, 0, None) == nat.DFS_ERR_UNSUPPORTED
    # a dense cost beyond the resident range streams C: a small workspace,
    # V head dims up to 128 (fp32), no backward
    dense = nat.make_problem(2, 3, 1000, 128, __import__("torch").float32, 5, 1.0, 10.0,
                             cost_mode=nat.DFS_COST_DENSE)
    assert lib.dfs_workspace_size(dense, ctypes.byref(fb), ctypes.byref(bb)) == nat.DFS_OK
    # the minimum: per-problem early-stop state (256 bytes here), then the transport's two row
    # statistics per point; dfs_dense_work_bytes more enables the one-read iterations (N <= 8192)
    r256 = lambda x: (x + 255) // 256 * 256  # noqa: E731
    assert fb.value == 256 + r256(2 * 6 * 1000 * 4) and bb.value == 0
    assert lib.dfs_dense_work_bytes(2, 3, 1000) == 148 * 8 * 2 * 1000 * 4
    fake_dense = nat.DfsFwdArgs(C=16, eps=16, log_mu=16, log_nu=16, log_u=16, log_v=16)
    assert lib.dfs_fwd(dense, fake_dense, None, 0, None) == nat.DFS_ERR_WORKSPACE
    wider = nat.make_problem(1, 1, 1000, 129, __import__("torch").float32, 5, 1.0, 10.0, cost_mode=nat.DFS_COST_DENSE)
    assert lib.dfs_fwd(wider, fake_dense, None, 0, None) == nat.DFS_ERR_UNSUPPORTED
    # a padded head dim needs its zero-padded copies even on the resident path:
    # Q, K, V (bf16) and O (fp32) at d = 32, each region rounded up to 256 bytes
    odd_d = nat.make_problem(2, 4, 16, 8, __import__("torch").bfloat16, 3, 1.0, 10.0)
    assert lib.dfs_fwd(odd_d, fake, None, 0, None) == nat.DFS_ERR_WORKSPACE
    assert lib.dfs_workspace_size(odd_d, ctypes.byref(fb), ctypes.byref(bb)) == nat.DFS_OK
    nd = 2 * 4 * 16 * 32
    assert fb.value == 3 * 2 * nd + 4 * nd  # already multiples of 256
    # backward: Q, K, V, dO, dQ, dK, dV copies, then the resident kernels' partials of
    # the shared-parameter gradients: dx (3 per point), dw, 68 bin sums and dr per CTA
    bh, cta = 2 * 4, 1
    assert bb.value == 3 * 2 * nd + 4 * 4 * nd + 4 * (bh * 16 * 3 + 2 * bh * cta + bh * cta * 68)
    # the phase API keeps no padded copies between calls
    assert lib.dfs_stream_op(nat.DFS_OP_FWD_INIT, odd_d, None, fake, None, 0, 16, None, 0, None) == \
        nat.DFS_ERR_UNSUPPORTED
    bad = nat.make_problem(1, 1, 64, 32, __import__("torch").bfloat16, 20, -1.0, 10.0)
    assert lib.dfs_fwd(bad, fake, None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    cg = nat.DfsCgParams(rtol=1e-6, atol=1e-6, max_iter=-1)
    ok = nat.make_problem(1, 1, 64, 32, __import__("torch").bfloat16, 20, 1.0, 10.0)
    assert lib.dfs_bwd(ok, cg, nat.DfsBwdArgs(), None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    fws, bws = ctypes.c_size_t(7), ctypes.c_size_t(7)
    assert lib.dfs_workspace_size(ok, ctypes.byref(fws), ctypes.byref(bws)) == nat.DFS_OK
    assert fws.value == 0
    assert lib.dfs_selftest_mma(5, None, None, None, 64, 32, 32, None) == nat.DFS_ERR_INVALID_ARGUMENT


def test_native_autograd_extension_loads():
    # dfsink_torch.so (csrc/dfs_torch.cpp) links libdfsink and carries the
    # autograd function behind flash_sinkhorn; importing it needs no GPU
    nat.build_torch_ext()
    ext = nat.ext()
    assert callable(ext.flash_sinkhorn) and callable(ext.last_report)
    assert ext.last_report() == []


def test_native_autograd_rejects_cpu_tensors():
    import torch

    ext = nat.ext()
    x = torch.zeros(1, 1, 64, 32)
    lm = torch.zeros(1, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ext.flash_sinkhorn(x, x, x, None, None, None, torch.ones(1), None, lm, lm, None, None, None,
                           5, float("inf"), 10.0, 1e-6, 0.0, 50)


def test_position_bin_arguments(lib):
    """pos_bins, or all three compute_bins inputs (chain_id, global_idx,
    bond_matrix), never both; dfs_compute_bins checks its pointers."""
    p = nat.make_problem(1, 2, 64, 32, __import__("torch").bfloat16, 5, float("inf"), 10.0)
    base = dict(Q=16, K=16, V=16, eps=16, log_mu=16, log_nu=16, log_u=16, log_v=16, pos_weight=16)
    assert lib.dfs_fwd(p, nat.DfsFwdArgs(**base), None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    part = nat.DfsFwdArgs(**base, chain_id=16, global_idx=16)
    assert lib.dfs_fwd(p, part, None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    both = nat.DfsFwdArgs(**base, pos_bins=16, chain_id=16, global_idx=16, bond_matrix=16)
    assert lib.dfs_fwd(p, both, None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    cg = nat.DfsCgParams(rtol=1e-6, atol=1e-6, max_iter=10)
    bwd = nat.DfsBwdArgs(Q=16, K=16, V=16, eps=16, log_mu=16, log_nu=16, log_u=16, log_v=16, dO=16,
                         pos_weight=16, dpos_weight=16, chain_id=16)
    assert lib.dfs_bwd(p, cg, bwd, None, 0, None) == nat.DFS_ERR_INVALID_ARGUMENT
    assert lib.dfs_compute_bins(2, 8, None, 16, 16, 16, None) == nat.DFS_ERR_INVALID_ARGUMENT
    assert lib.dfs_compute_bins(-1, 8, 16, 16, 16, 16, None) == nat.DFS_ERR_INVALID_ARGUMENT
    assert lib.dfs_compute_bins(0, 8, None, None, None, None, None) == nat.DFS_OK


def test_dense_gradient_entry_points_validate_on_the_host(lib):
    """The dense-gradient calls reject bad sizes and missing buffers before any
    device work (no GPU needed)."""
    E = nat.DFS_ERR_INVALID_ARGUMENT
    p = 256  # any non-null, 16-byte aligned address: nothing is dereferenced on these paths

    def it(B, H, N, lam, hist, i0, i1, work):
        return lib.dfs_dense_iterate(B, H, N, lam, p, p, p, p, None, None, None, hist, i0, i1, p, p, None, work,
                                     None, None)
    assert it(0, 1, 8, 1.0, p, 0, 1, p) == E
    assert it(1, 1, 8, 1.0, p, 2, 1, p) == E
    assert it(1, 1, 1 << 17, 1.0, p, 0, 1, p) == E
    assert it(1, 1, 8, 0.0, p, 0, 1, p) == E
    assert it(1, 1, 8, 1.0, None, 0, 1, p) == E
    assert it(1, 1, 8, 1.0, p, 0, 1, None) == E        # N <= 8192 needs the work buffer
    assert it(1, 1, 8, 1.0, p, 0, 1, p + 4) == E       # ... 16-byte aligned
    assert lib.dfs_dense_work_bytes(2, 3, 100) == 148 * 8 * 2 * 100 * 4
    assert lib.dfs_dense_work_bytes(1, 1, 9000) == 0
    assert lib.dfs_dense_solve_bwd(1, 1, 8, -1, 1.0, p, p, p, p, None, p, None, None, None, None, None, None, None,
                                   p, None) == E
    assert lib.dfs_dense_solve_bwd(1, 1, 8, 3, 1.0, p, p, p, p, None, p, None, None, None, None, None, None, None,
                                   None, None) == E
    assert lib.dfs_dense_transport_bwd(1, 0, 8, p, p, p, None, None) == E
    assert lib.dfs_dense_transport_bwd(1, 1, 8, None, p, p, None, None) == E


def test_dense_backward_scratch_size(lib):
    """(7 iters + 5) slots of B*H*N floats rounded up to 64, 4 floats per
    (batch, head) rounded up to 64, and for N <= 8192 the one-read reverse
    iterations' column sums (N floats for up to max(B*H, 148 x 8) CTAs); 0 for
    invalid sizes."""
    assert lib.dfs_dense_solve_bwd_scratch(1, 1, 8, 3) == ((7 * 3 + 5) * 64 + 64 + 1184 * 8) * 4
    assert lib.dfs_dense_solve_bwd_scratch(2, 3, 100, 20) == ((7 * 20 + 5) * 640 + 64 + 1184 * 100) * 4
    assert lib.dfs_dense_solve_bwd_scratch(1, 1, 9000, 2) == ((7 * 2 + 5) * 9024 + 64) * 4
    assert lib.dfs_dense_solve_bwd_scratch(0, 1, 8, 3) == 0
    assert lib.dfs_dense_solve_bwd_scratch(1, 1, 8, -1) == 0
