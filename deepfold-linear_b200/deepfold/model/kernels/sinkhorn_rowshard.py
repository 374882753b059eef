"""Row-sharded flash Sinkhorn: one long-sequence problem set over several GPUs.

The long-sequence configuration (B=1, H=16, N=8192, d=64) splits the query rows of every
(batch, head) problem evenly over the GPUs of a ``torch.distributed`` group
(NCCL over NVLink).  Every GPU holds Q, K, V, dO and the marginals in full
(N x d per head: a few MB) and owns one contiguous range of rows, which is also
its range of columns for the column half-updates (the streamed kernels run a
column update as a row update of S^T = K Q^T).  Each phase of the streamed
path (``dfs_stream_op`` in include/dfsink.h) runs on the local range, and the
vectors a phase produced are all-gathered before the next one:

* forward: per Sinkhorn iteration the row potential f after the row half-update
  and the column potential g after the column half-update (B*H*N fp32 each);
* backward: the row statistics, the column sums, and per CG iteration the two
  matrix-free plan products t = D1^-1 P u and s = P^T t; the CG scalars are then
  computed redundantly, and identically, on every GPU, so all GPUs stop the
  solve together without a further collective.

Outputs (O, potentials, gradients) are all-gathered too, so every rank ends
with the same full tensors a single GPU would produce.

On NCCL groups whose shapes the TMA-staged kernels cover, the forward's
half-updates exchange their potentials without any collective: each rank's
forward workspace is a device buffer shared with the other ranks through CUDA
IPC (``_PeerWorkspace``), and the half-update kernel stores its rows of the new
potential straight into every rank's copy over NVLink and raises every rank's
arrival counter; the next half-update waits on its own counter
(``dfs_stream_op_peer``).  The backward's workspace is shared the same way,
and its row statistics, column sums and CG vectors are gathered through peer
memory too (``dfs_peer_gather_rows``: every rank pushes its rows into every
other rank's copy, raises their counters, and waits on its own), and so are
dQ, dK, dV (written into a third shared buffer, gathered, copied out): no
collective on the data path.  ``DFS_ROWSHARD_EXCHANGE=collective`` selects the
all-gather exchange for both instead.  Where the reference
runs on one device only (src/deepfold/model/kernels/sinkhorn_kernel.py), this
module has no counterpart there.
"""

from __future__ import annotations

import ctypes
import math
import os

import torch
import torch.distributed as dist

from deepfold import _native as nat

__all__ = ["row_range", "RowGather", "arrivals_per_half_update", "row_sharded_flash_sinkhorn",
           "last_rowshard_report"]


def row_range(N: int, world: int, rank: int) -> tuple[int, int, int]:
    """Rows [r0, r1) of `rank` and the padded per-rank length ceil(N / world)."""
    n_loc = -(-N // world)
    r0 = min(N, rank * n_loc)
    return r0, min(N, r0 + n_loc), n_loc


class RowGather:
    """All-gather of row slices: each rank holds valid rows [r0, r1) of a tensor
    (P, N, *rest) laid out like the kernels' (B*H, N, ...) vectors; after the
    call every rank holds all rows."""

    def __init__(self, N: int, group=None):
        self.group = group
        on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if on else 1
        self.rank = dist.get_rank(group) if on else 0
        self.nccl = on and dist.get_backend(group) == "nccl"
        self.N = N
        self.r0, self.r1, self.n_loc = row_range(N, self.world, self.rank)

    def _buffers(self, x: torch.Tensor):
        """The send and receive buffers for tensors of x's shape, kept for the
        process's lifetime: the same addresses every call, so no call allocates
        (the backward gathers 33 MB gradients; a fresh allocation can stall a rank
        on the host while the others wait in the collective).  Stream order makes
        reuse safe: a gather's copies are queued before the next gather."""
        key = (tuple(x.shape), x.dtype, x.device, self.world, self.rank, id(self.group))
        buf = _gather_bufs.get(key)
        if buf is None:
            P, rest = x.shape[0], tuple(x.shape[2:])
            buf = (x.new_zeros((P, self.n_loc) + rest), x.new_empty((self.world, P, self.n_loc) + rest))
            _gather_bufs[key] = buf
        return buf

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        loc, out = self._buffers(x)
        loc[:, : self.r1 - self.r0] = x[:, self.r0:self.r1]  # rows past r1 (uneven split) stay zero
        if self.nccl:
            dist.all_gather_into_tensor(out, loc, group=self.group)
        else:  # gloo (CPU tests of this orchestration)
            dist.all_gather(list(out.unbind(0)), loc, group=self.group)
        # rank r's rows land at [r n_loc, min(N, (r + 1) n_loc)): one strided copy each
        for r in range(self.world):
            a = min(self.N, r * self.n_loc)
            b = min(self.N, a + self.n_loc)
            if b > a:
                x[:, a:b].copy_(out[r, :, : b - a])
        return x


_gather_bufs: dict = {}


def arrivals_per_half_update(P: int, N: int, world: int) -> int:
    """Counter arrivals one peer-exchange half-update raises on every rank: each
    rank's kernel signals once per block of 128 rows of each of the P problems
    in its row range (the column-split CTAs of a block signal once, through the
    block's last CTA)."""
    total = 0
    for r in range(world):
        r0, r1, _ = row_range(N, world, r)
        total += P * (-(-(r1 - r0) // 128))
    return total


class _PeerWorkspace:
    """This rank's forward workspace, shared with every rank of the group through
    CUDA IPC (allocated zero-filled by the library, handles all-gathered over
    the group), and the cumulative count of arrivals its counter has been told
    to expect -- identical on every rank, since all ranks run the same phases."""

    def __init__(self, nbytes: int, group, device: torch.device):
        L = nat.lib()
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        p, h = ctypes.c_void_p(), nat.DfsIpcHandle()
        nat.check(L.dfs_peer_alloc(nbytes, ctypes.byref(p), ctypes.byref(h)), "dfs_peer_alloc")
        self.ptr = p.value
        mine = torch.tensor(list(bytes(h.bytes)), dtype=torch.uint8, device=device)
        every = torch.empty(self.world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().tolist()
        self.ws = []
        for r in range(self.world):
            if r == self.rank:
                self.ws.append(self.ptr)
                continue
            hr = nat.DfsIpcHandle()
            for i, v in enumerate(every[64 * r:64 * (r + 1)]):
                hr.bytes[i] = v
            q = ctypes.c_void_p()
            nat.check(L.dfs_peer_open(ctypes.byref(hr), ctypes.byref(q)), "dfs_peer_open")
            self.ws.append(q.value)
        self.arrived = 0
        self.peers = nat.DfsPeerSet(npeers=self.world, self=self.rank)
        for k, w in enumerate(self.ws):
            self.peers.ws[k] = w


_peer_ws: dict = {}


def _peer_workspace(nbytes: int, group, device: torch.device, kind: str = "fwd") -> _PeerWorkspace:
    key = (kind, nbytes, device.index, id(group))
    if key not in _peer_ws:
        with torch.cuda.device(device):  # the buffer and the peer mappings belong to this GPU
            _peer_ws[key] = _PeerWorkspace(nbytes, group, device)
    return _peer_ws[key]


class _CudaFloats:
    """A device buffer the library allocated, described for torch.as_tensor
    (the CUDA array interface): a float32 vector of n elements at ptr."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def _device_floats(ptr: int, n: int, device: torch.device) -> torch.Tensor:
    """A torch view (no copy) of n float32 at ptr on `device`, valid while the
    buffer lives (peer workspaces live until the process exits)."""
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaFloats(ptr, n), device=device)


def _slot(ws: torch.Tensor, k: int, P: int, N: int) -> torch.Tensor:
    return ws[k * P * N:(k + 1) * P * N].view(P, N)


class _Sharded:
    """One row-sharded problem set: argument blocks, workspaces and the phase loop."""

    def __init__(self, Q, K, V, eps, log_mu, log_nu, K_iter, lam, mask, log_u_init, log_v_init, x_res,
                 cg, group):
        nat.require_cuda(Q, K, V)
        self.B, self.H, self.N, self.d = Q.shape
        self.P = self.B * self.H
        self.group = group
        self.gather = RowGather(self.N, group)
        cdt = Q.dtype if Q.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
        f32 = lambda t: None if t is None else t.contiguous().float()  # noqa: E731
        self.Q, self.K, self.V = (t.contiguous().to(cdt) for t in (Q, K, V))
        self.eps, self.lmu, self.lnu = f32(eps), f32(log_mu), f32(log_nu)
        self.mask, self.lui, self.lvi, self.xr = f32(mask), f32(log_u_init), f32(log_v_init), f32(x_res)
        self.K_iter, self.lam, self.cg = int(K_iter), float(lam), cg
        self.prob = nat.make_problem(self.B, self.H, self.N, self.d, cdt, K_iter, lam, 10.0)
        self.fwd_bytes, self.bwd_bytes = nat.workspace_bytes(self.prob)
        self.stream = nat.stream_ptr(Q.device)

    def _op(self, op, r0, r1, fa=None, ba=None, ws=None, nbytes=0, cgp=None):
        nat.check(nat.lib().dfs_stream_op(op, self.prob, cgp, fa, ba, r0, r1, ws.data_ptr(), nbytes,
                                          self.stream), f"dfs_stream_op({op})")

    def forward(self):
        dev = self.Q.device
        B, H, N, d, P = self.B, self.H, self.N, self.d, self.P
        fo = dict(device=dev, dtype=torch.float32)
        self.O = torch.empty(B, H, N, d, **fo)
        self.xc = torch.empty(B, H, N, 3, **fo) if self.xr is not None else None
        self.lu, self.lv = torch.empty(B, H, N, **fo), torch.empty(B, H, N, **fo)
        self.fstatus = torch.zeros(1, device=dev, dtype=torch.int32)
        peer = self._peer_exchange()
        outs = [self.O, self.lu, self.lv] + ([self.xc] if self.xc is not None else [])
        widths = [d, 1, 1, 3]
        if peer:
            # the phases write O, log_u, log_v (x_centroid) into a buffer shared with
            # every rank; their rows are gathered through peer memory and copied out
            sizes = [P * N * w for w in widths[:len(outs)]]
            offs = [sum(sizes[:k]) for k in range(len(sizes))]
            fcnt_off = -(-sum(sizes) * 4 // 256) * 256
            pwo = _peer_workspace(fcnt_off + 256, self.group, dev, kind="fout")
            flat = _device_floats(pwo.ptr, sum(sizes), dev)
            kouts = [flat[o:o + n].view(t.shape) for o, n, t in zip(offs, sizes, outs)]
        else:
            kouts = outs
        kO, klu, klv = kouts[0], kouts[1], kouts[2]
        kxc = kouts[3] if self.xc is not None else None
        fa = nat.DfsFwdArgs(Q=nat.ptr(self.Q), K=nat.ptr(self.K), V=nat.ptr(self.V), x_res=nat.ptr(self.xr),
                            eps=nat.ptr(self.eps), log_mu=nat.ptr(self.lmu), log_nu=nat.ptr(self.lnu),
                            log_u_init=nat.ptr(self.lui), log_v_init=nat.ptr(self.lvi), mask=nat.ptr(self.mask),
                            O=nat.ptr(kO), x_centroid=nat.ptr(kxc), log_u=nat.ptr(klu),
                            log_v=nat.ptr(klv), status=nat.ptr(self.fstatus))
        g, r0, r1 = self.gather, self.gather.r0, self.gather.r1
        if peer:
            self._forward_peer(fa, r0, r1)
            for k, (t, kt) in enumerate(zip(outs, kouts)):
                nat.check(nat.lib().dfs_peer_gather_rows(pwo.peers, offs[k] * 4, P, N, widths[k], r0, r1, fcnt_off,
                                                         nat.ptr(self.fstatus), self.stream), "dfs_peer_gather_rows")
                t.copy_(kt)
            return self.O, self.xc, self.lu, self.lv
        else:
            ws = torch.empty(max(self.fwd_bytes // 4, 1), **fo)
            run = lambda op, a, b: self._op(op, a, b, fa=fa, ws=ws, nbytes=self.fwd_bytes)  # noqa: E731
            run(nat.DFS_OP_FWD_INIT, 0, N)
            f, gg = _slot(ws, nat.DFS_WS_FWD_F, P, N), _slot(ws, nat.DFS_WS_FWD_G, P, N)
            for _ in range(self.K_iter):
                run(nat.DFS_OP_FWD_ROWS, r0, r1)
                g(f)
                run(nat.DFS_OP_FWD_COLS, r0, r1)
                g(gg)
            run(nat.DFS_OP_FWD_OUT, r0, r1)
        if self.K_iter > 0:
            g(self.lu.view(P, N))
            g(self.lv.view(P, N))
        g(self.O.view(P, N, d))
        if self.xc is not None:
            g(self.xc.view(P, N, 3))
        return self.O, self.xc, self.lu, self.lv

    def _peer_exchange(self) -> bool:
        """Half-updates exchange their potentials through peer memory (NCCL group of
        several GPUs, shapes on the TMA-staged kernels) unless disabled."""
        g = self.gather
        if g.world < 2 or not g.nccl or os.environ.get("DFS_ROWSHARD_EXCHANGE", "peer") != "peer":
            return False
        tma = (self.d == 64 or (self.d == 32 and self.Q.dtype == torch.float32)) and self.N >= 128
        return tma and g.world <= nat.DFS_MAX_PEERS

    def _forward_peer(self, fa, r0, r1):
        """The forward's phase loop with the peer exchange (every rank in lockstep).
        (Two interleaved problem groups, so that one group's exchange hides behind
        the other's half-update, measured slower on 2 and 4 GPUs at N = 8192: the
        halved grids cost more than the waits they hide.)"""
        pw = _peer_workspace(self.fwd_bytes, self.group, self.Q.device)
        L = nat.lib()
        world = self.gather.world
        blocks = arrivals_per_half_update(self.P, self.N, world)

        def run(op, a, b, wait):
            pw.peers.wait_for = wait
            nat.check(L.dfs_stream_op_peer(op, self.prob, fa, a, b, pw.ptr, self.fwd_bytes, pw.peers,
                                           self.stream), f"dfs_stream_op_peer({op})")

        run(nat.DFS_OP_FWD_INIT, 0, self.N, 0)
        pw.arrived += world  # every rank's init raised every counter once
        for _ in range(self.K_iter):
            run(nat.DFS_OP_FWD_ROWS, r0, r1, pw.arrived)
            pw.arrived += blocks
            run(nat.DFS_OP_FWD_COLS, r0, r1, pw.arrived)
            pw.arrived += blocks
        run(nat.DFS_OP_FWD_OUT, r0, r1, pw.arrived)

    def backward(self, dO, dxc, need_marg: bool):
        dev = self.Q.device
        B, H, N, d, P = self.B, self.H, self.N, self.d, self.P
        fo = dict(device=dev, dtype=torch.float32)
        dOc = dO.contiguous().float()
        dxcc = None if (dxc is None or self.xr is None) else dxc.contiguous().float()
        dQ, dK, dV = (torch.empty(B, H, N, d, **fo) for _ in range(3))
        peer = self._peer_exchange()
        if peer:
            # the gradient passes write into a buffer shared with every rank, whose
            # rows are then gathered through peer memory and copied out
            gbytes = 3 * P * N * d * 4
            gcnt_off = -(-gbytes // 256) * 256
            pwg = _peer_workspace(gcnt_off + 256, self.group, dev, kind="grad")
            gview = _device_floats(pwg.ptr, 3 * P * N * d, dev).view(3, B, H, N, d)
            kQ, kK, kV = gview[0], gview[1], gview[2]
        else:
            kQ, kK, kV = dQ, dK, dV
        dmu = torch.empty(B, H, N, **fo) if need_marg else None
        dnu = torch.empty(B, H, N, **fo) if need_marg else None
        iters = torch.empty(P, device=dev, dtype=torch.int32)
        resid = torch.empty(P, **fo)
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        if peer:
            # the workspace is shared with every rank (CUDA IPC); its slot gathers
            # go through peer memory, the arrival counters after the workspace
            cnt_off = -(-self.bwd_bytes // 256) * 256
            pwb = _peer_workspace(cnt_off + 256, self.group, dev, kind="bwd")
            ws = _device_floats(pwb.ptr, max(self.bwd_bytes // 4, 1), dev)
        else:
            ws = torch.empty(max(self.bwd_bytes // 4, 1), **fo)
        cgp = nat.DfsCgParams(rtol=float(self.cg["rtol"]), atol=float(self.cg["atol"]),
                              max_iter=int(self.cg["max_iter"]), reserved=0)
        ba = nat.DfsBwdArgs(Q=nat.ptr(self.Q), K=nat.ptr(self.K), V=nat.ptr(self.V), x_res=nat.ptr(self.xr),
                            eps=nat.ptr(self.eps), log_mu=nat.ptr(self.lmu), log_nu=nat.ptr(self.lnu),
                            mask=nat.ptr(self.mask), log_u=nat.ptr(self.lu), log_v=nat.ptr(self.lv),
                            dO=nat.ptr(dOc), dxc=nat.ptr(dxcc), dQ=nat.ptr(kQ), dK=nat.ptr(kK), dV=nat.ptr(kV),
                            dlog_mu=nat.ptr(dmu), dlog_nu=nat.ptr(dnu), cg_iters=nat.ptr(iters),
                            cg_residual=nat.ptr(resid), status=nat.ptr(status))
        g, r0, r1 = self.gather, self.gather.r0, self.gather.r1
        run = lambda op, a=0, b=N: self._op(op, a, b, ba=ba, ws=ws, nbytes=self.bwd_bytes, cgp=cgp)  # noqa: E731
        slot = lambda k: _slot(ws, k, P, N)  # noqa: E731

        def gslot(k):
            """Every rank's rows of workspace slot k on every rank."""
            if not peer:
                g(slot(k))
                return
            # every rank runs the same gathers in the same order: the waits count on the device
            nat.check(nat.lib().dfs_peer_gather_rows(pwb.peers, k * P * N * 4, P, N, 1, r0, r1, cnt_off,
                                                     nat.ptr(status), self.stream), "dfs_peer_gather_rows")
        # the per-problem CG stop flags (int32) follow the vector slots and the scalars
        o = nat.DFS_WS_BWD_NSLOTS * P * N + nat.DFS_WS_BWD_NSCALARS * P
        done = ws[o:o + P].view(torch.int32)
        run(nat.DFS_OP_BWD_PREP)
        run(nat.DFS_OP_BWD_ROWSTATS, r0, r1)
        for k in (nat.DFS_WS_BWD_M, nat.DFS_WS_BWD_R, nat.DFS_WS_BWD_D):
            gslot(k)
        run(nat.DFS_OP_BWD_ROWDERIVE)
        run(nat.DFS_OP_BWD_COLSTATS, r0, r1)
        gslot(nat.DFS_WS_BWD_C)
        gslot(nat.DFS_WS_BWD_GV)
        run(nat.DFS_OP_BWD_SETUP)
        run(nat.DFS_OP_BWD_PT_T, r0, r1)
        gslot(nat.DFS_WS_BWD_S)
        run(nat.DFS_OP_BWD_CGINIT)
        # The stop flags are identical on every rank (same gathered vectors, same
        # arithmetic), so all ranks leave the loop after the same iteration.  The
        # host reads them one iteration late: iteration k is queued before the
        # flags of k - 1 are tested, so the GPU never idles on that read; the one
        # extra iteration after convergence skips every converged problem (its
        # plan products and CG step return at once).
        stream = torch.cuda.current_stream(dev)
        first_round = 0
        if peer:
            # round 0 phase by phase, then every later round inside one graph whose
            # loop stops on the device: no host read of the stop flags at all
            run(nat.DFS_OP_BWD_P_U, r0, r1)
            gslot(nat.DFS_WS_BWD_T)
            run(nat.DFS_OP_BWD_PT_T, r0, r1)
            gslot(nat.DFS_WS_BWD_S)
            run(nat.DFS_OP_BWD_CGSTEP_FIRST)
            rc = nat.lib().dfs_stream_cg_loop_peer(self.prob, cgp, ba, r0, r1, ws.data_ptr(), self.bwd_bytes,
                                                   pwb.peers, cnt_off, self.stream)
            if rc == nat.DFS_OK:
                first_round = None
            elif rc == nat.DFS_ERR_UNSUPPORTED:
                first_round = 1  # no conditional graphs here: the host loop below from round 1
            else:
                nat.check(rc, "dfs_stream_cg_loop_peer")
        flag_bufs, flag_evs = _flag_buffers(P, dev)
        pending = None
        for it in (range(first_round, int(self.cg["max_iter"]) + 1) if first_round is not None else ()):
            run(nat.DFS_OP_BWD_P_U, r0, r1)
            gslot(nat.DFS_WS_BWD_T)
            run(nat.DFS_OP_BWD_PT_T, r0, r1)
            gslot(nat.DFS_WS_BWD_S)
            run(nat.DFS_OP_BWD_CGSTEP_FIRST if it == 0 else nat.DFS_OP_BWD_CGSTEP)
            buf, ev = flag_bufs[it & 1], flag_evs[it & 1]
            buf.copy_(done, non_blocking=True)
            ev.record(stream)
            prev, pending = pending, (ev, buf)
            if prev is not None:
                prev[0].synchronize()
                if bool((prev[1] != 0).all()):
                    break
        run(nat.DFS_OP_BWD_P_X, r0, r1)
        gslot(nat.DFS_WS_BWD_S)
        run(nat.DFS_OP_BWD_FINAL)
        run(nat.DFS_OP_BWD_DQ, r0, r1)
        run(nat.DFS_OP_BWD_DKV, r0, r1)
        if peer:
            for k, t in enumerate((dQ, dK, dV)):
                nat.check(nat.lib().dfs_peer_gather_rows(pwg.peers, k * P * N * d * 4, P, N, d, r0, r1, gcnt_off,
                                                         nat.ptr(status), self.stream), "dfs_peer_gather_rows")
                t.copy_(gview[k])
        else:
            for t in (dQ, dK, dV):
                g(t.view(P, N, d))
        self.report = dict(cg_iters=iters, cg_residual=resid, status=status, fwd_status=self.fstatus)
        _last_report.clear()
        _last_report.update(self.report)
        return dQ, dK, dV, dmu, dnu


_last_report: dict = {}
_flag_cache: dict = {}


def _flag_buffers(P: int, device: torch.device):
    """Two pinned host buffers for the CG stop flags and two events, made once per
    (P, device): pinning host memory inside a timed loop can stall the host for
    milliseconds, and every rank waits for a stalled one.  Reuse is ordered by
    the stream: a buffer is read only after the event of its own copy."""
    key = (P, device.index)
    if key not in _flag_cache:
        _flag_cache[key] = ([torch.empty(P, dtype=torch.int32).pin_memory() for _ in range(2)],
                            [torch.cuda.Event() for _ in range(2)])
    return _flag_cache[key]


def last_rowshard_report() -> dict:
    """Device tensors (cg_iters, cg_residual, status, fwd_status) of the most
    recent row-sharded backward on this rank."""
    return dict(_last_report)


class _RowShardedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, log_mu, log_nu, eps, mask, x_res, K_iter, lam, cg, group):
        sh = _Sharded(Q, K, V, eps, log_mu, log_nu, K_iter, lam, mask, None, None, x_res, cg, group)
        O, xc, lu, lv = sh.forward()
        ctx.sh = sh
        ctx.in_dtype = Q.dtype
        ctx.mark_non_differentiable(lu, lv)
        if xc is None:
            xc = O.new_zeros(0)
        return O, xc, lu, lv

    @staticmethod
    def backward(ctx, dO, dxc, _dlu, _dlv):
        sh = ctx.sh
        need_marg = ctx.needs_input_grad[3] or ctx.needs_input_grad[4]
        if dO is None:
            dO = torch.zeros_like(sh.O)
        dQ, dK, dV, dmu, dnu = sh.backward(dO, dxc if sh.xr is not None else None, need_marg)
        cast = lambda t: t.to(ctx.in_dtype)  # noqa: E731
        return (cast(dQ), cast(dK), cast(dV), dmu, dnu, None, None, None, None, None, None, None)


def row_sharded_flash_sinkhorn(Q, K, V, eps, log_mu, log_nu, K_iter: int = 7, lam: float = 1.0, mask=None,
                               x_res=None, cg_opts: dict | None = None, group=None):
    """flash_sinkhorn (sinkhorn_kernel.flash_sinkhorn) with the rows of every
    problem split over the ranks of `group`.  Every rank passes the same full
    (B, H, N, d) inputs and receives the same full outputs (O, x_centroid or
    None, log_u, log_v); backward gives the full gradients on every rank.
    Uses the streamed kernels (d = 32 or 64; no position / geometry terms)."""
    from deepfold.model.kernels.sinkhorn_kernel import CG_DEFAULTS

    cg = dict(CG_DEFAULTS)
    if cg_opts:
        cg.update(cg_opts)
    if not (lam > 0.0) or math.isnan(lam):
        raise ValueError("lam must be positive (inf for the balanced problem)")
    O, xc, lu, lv = _RowShardedFn.apply(Q, K, V, log_mu, log_nu, eps, mask, x_res, int(K_iter), float(lam), cg,
                                        group)
    return O, (xc if x_res is not None else None), lu, lv
