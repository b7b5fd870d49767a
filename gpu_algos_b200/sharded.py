"""Observation-sharded GLM gradient and elastic-net fit across ranks.

The reference is single-GPU.  Here the observations are split into
contiguous blocks, one per rank (one process per GPU, ``torch.distributed``
for the plumbing): every rank evaluates

    P_r = sum_{obs in block r} (Yhat - Y) X          (float64, no factor 2)

with the fused kernel (``glmb_gradient_partial_*``), the P_r are summed with
ONE all-reduce, and every rank applies the same finalize step, so all ranks
hold bit-identical gradients / coefficients.  Tasks shard with no collective
at all (each task's gradient only involves its own observations), which is
what :func:`task_range` is for.

The per-rank arithmetic goes through a :class:`Backend`: :class:`CudaBackend`
calls ``libglm_b200.so``; the CPU tests supply their own backend and run the
same orchestration on ``gloo`` ranks.

Two exchanges are available: :class:`CudaBackend` sums the rank partials
with one NCCL all-reduce; :class:`PeerBackend` does the sum inside the
library, over NVLink peer memory (``glmb_gradient_sharded_*``: the partial
kernel plus one exchange kernel, no collective library on the path).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

#: safety factor applied to the power-iteration estimate of the Lipschitz constant
POWER_SAFETY = 1.05


def obs_range(nobs: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block [lo, hi) of observations owned by ``rank``; the
    first ``nobs % world`` ranks hold one extra observation."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(nobs, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def task_range(ntasks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block [lo, hi) of tasks owned by ``rank`` (task sharding)."""
    return obs_range(ntasks, world, rank)


class Backend:
    """Per-rank arithmetic of the sharded path (all tensors on one device)."""

    def partial(self, X, M, Y):  # -> float64 (ntasks, nt, nf)
        raise NotImplementedError

    def finalize(self, P, M, lam, alpha, out):  # grad = 2P + elastic-net term
        raise NotImplementedError

    def power_init(self, v, seed):
        raise NotImplementedError

    def power_step(self, P, v, norm, lipschitz, lambda2):
        raise NotImplementedError

    def prox_update(self, P, beta, lipschitz, lambda1, lambda2):
        raise NotImplementedError

    # Full-data results.  The default is the local partial followed by an
    # all-reduce over `group`; a backend that exchanges by itself overrides them.
    def reduced_partial(self, X, M, Y, group):
        return _all_reduce(self.partial(X, M, Y), group)

    def reduced_gradient(self, X, M, Y, lam, alpha, out, group):
        return self.finalize(self.reduced_partial(X, M, Y, group), M, lam, alpha, out)


class CudaBackend(Backend):
    """The sm_100a kernels of libglm_b200.so."""

    def __init__(self, workspace=None):
        from . import glm

        self.glm = glm
        self.workspace = workspace

    def partial(self, X, M, Y, out=None):
        return self.glm.gradient_partial(X, M, Y, out=out, workspace=self.workspace)

    def finalize(self, P, M, lam, alpha, out):
        return self.glm.gradient_finalize(P, M, lam, alpha, True, out=out)

    def power_init(self, v, seed):
        return self.glm.power_init(v, seed)

    def power_step(self, P, v, norm, lipschitz, lambda2):
        return self.glm.power_step(P, v, norm, lipschitz, lambda2)

    def prox_update(self, P, beta, lipschitz, lambda1, lambda2):
        return self.glm.prox_update(P, beta, lipschitz, lambda1, lambda2)


class PeerGroup:
    """This rank's member of a library peer-exchange group.

    Creates the rank's exchange buffer, all-gathers the buffers' IPC handles
    over ``group`` (the only use of torch.distributed) and maps the peers'
    buffers.  ``max_elems`` bounds nfeatures*ntargets*ntasks of the
    gradients exchanged; ``timeout_ms`` bounds every wait for a peer.
    """

    def __init__(self, max_elems: int, timeout_ms: float = 2000.0, group=None):
        from . import capi

        self.capi = capi
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        handle = ctypes.create_string_buffer(capi.PEER_HANDLE_BYTES)
        ptr = ctypes.c_void_p()
        capi.call("glmb_peer_group_create", self.rank, self.world, int(max_elems), float(timeout_ms),
                  ctypes.byref(ptr), handle)
        self.ptr = ptr
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        blob = ctypes.create_string_buffer(b"".join(handles), capi.PEER_HANDLE_BYTES * self.world)
        capi.call("glmb_peer_group_connect", self.ptr, blob)

    def status(self, reset: bool = True) -> int:
        """0, or 1 when a wait for a peer ran out (the call's outputs are NaN)."""
        st = ctypes.c_int(0)
        self.capi.call("glmb_peer_group_status", self.ptr, ctypes.byref(st), int(reset))
        return st.value

    def close(self):
        if self.ptr is not None:
            self.capi.call("glmb_peer_group_destroy", self.ptr)
            self.ptr = None


class PeerBackend(CudaBackend):
    """CudaBackend whose cross-rank sum runs over NVLink peer memory inside
    the library (one exchange kernel per evaluation)."""

    def __init__(self, peer: PeerGroup, workspace=None):
        super().__init__(workspace)
        self.peer = peer

    def _sharded(self, X, M, Y, grad, partial, lam, alpha, regularize):
        from . import capi, glm

        sfx = glm.SUFFIX[X.dtype]
        nobs, ntasks, nf = X.shape
        nt = M.shape[1]
        flags = capi.GRAD_REGULARIZE if regularize else 0
        if Y is None:
            flags |= capi.GRAD_Y_ZERO
        ws_ptr, ws_bytes = ((None, 0) if self.workspace is None
                            else (self.workspace.data_ptr(), self.workspace.numel() * self.workspace.element_size()))
        capi.call(f"glmb_gradient_sharded_{sfx}", X.data_ptr(), M.data_ptr(), None if Y is None else Y.data_ptr(),
                  None if grad is None else grad.data_ptr(), None if partial is None else partial.data_ptr(), None,
                  nf, nt, ntasks, nobs, float(lam), float(alpha), flags, self.peer.ptr, ws_ptr, ws_bytes,
                  torch.cuda.current_stream().cuda_stream)

    def reduced_partial(self, X, M, Y, group, out=None):
        ntasks, nt, nf = M.shape
        if out is None:
            out = torch.empty((ntasks, nt, nf), dtype=torch.float64, device=X.device)
        self._sharded(X, M, Y, None, out, 0.0, 0.0, False)
        return out

    def reduced_gradient(self, X, M, Y, lam, alpha, out, group):
        self._sharded(X, M, Y, out, None, lam, alpha, True)
        return out

    def fit(self, X, Y, lambda1, lambda2, n_power, n_iter, seed, beta=None, lipschitz=None):
        """The whole sharded fit in one library call (glmb_fit_elastic_net_sharded_*):
        the power iterations and ISTA steps, each partial summed over the group."""
        from . import capi, glm

        sfx = glm.SUFFIX[X.dtype]
        nobs, ntasks, nf = X.shape
        nt = Y.shape[2]
        if beta is None:
            beta = torch.empty((ntasks, nt, nf), dtype=X.dtype, device=X.device)
        if lipschitz is None:
            lipschitz = torch.empty((ntasks,), dtype=torch.float64, device=X.device)
        need = int(getattr(capi.lib(), f"glmb_fit_workspace_size_{sfx}")(nf, nt, ntasks, nobs))
        ws = self.workspace
        if ws is None or ws.numel() * ws.element_size() < need:
            ws = torch.empty(max(need, 1), dtype=torch.uint8, device=X.device)
        capi.call(f"glmb_fit_elastic_net_sharded_{sfx}", X.data_ptr(), Y.data_ptr(), beta.data_ptr(),
                  lipschitz.data_ptr(), nf, nt, ntasks, nobs, float(lambda1), float(lambda2), int(n_power),
                  int(n_iter), int(seed) & (2**64 - 1), self.peer.ptr, ws.data_ptr(),
                  ws.numel() * ws.element_size(), torch.cuda.current_stream().cuda_stream)
        return beta, lipschitz


def _all_reduce(t, group):
    if group is not None or (dist.is_available() and dist.is_initialized()):
        if dist.get_world_size(group) > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


@dataclass
class ShardedGLM:
    """This rank's block of observations and the collective that joins them.

    X_local: (nobs_local, ntasks, nf), Y_local: (nobs_local, ntasks, nt).
    Every rank must make the same sequence of calls (they all take part in
    each all-reduce).
    """

    X_local: torch.Tensor
    Y_local: torch.Tensor
    backend: Backend
    group: object = None

    def partial_sum(self, M, Y=None, y_zero=False):
        return self.backend.reduced_partial(self.X_local, M, None if y_zero else (self.Y_local if Y is None else Y),
                                            self.group)

    def gradient(self, M, lam: float, alpha: float, out=None):
        """Full-data gradient 2 sum (Yhat - Y) X + lam(alpha sign M + 2(1-alpha) M)."""
        if out is None:
            out = torch.empty_like(M)
        return self.backend.reduced_gradient(self.X_local, M, self.Y_local, lam, alpha, out, self.group)

    def fit_elastic_net(self, lambda1: float, lambda2: float, n_power: int = 20, n_iter: int = 200,
                        seed: int = 42, checkpoint=None, resume=None):
        """ISTA on the sharded data: returns (beta, lipschitz per task).

        ``checkpoint(it, beta, lipschitz)`` (optional) is called after every
        iteration on every rank; ``resume=(it, beta, lipschitz)`` restarts
        from a snapshot taken that way (skipping the power iteration).
        """
        if checkpoint is None and resume is None and hasattr(self.backend, "fit"):
            # the library runs the whole loop (PeerBackend)
            return self.backend.fit(self.X_local, self.Y_local, lambda1, lambda2, n_power, n_iter, seed)
        ntasks, nf = self.X_local.shape[1], self.X_local.shape[2]
        nt = self.Y_local.shape[2]
        dev, dt = self.X_local.device, self.X_local.dtype
        if resume is not None:
            start, beta0, lip0 = resume
            beta = beta0.clone().to(dev)
            lipschitz = lip0.clone().to(dev)
        else:
            start = 0
            v = torch.empty((ntasks, 1, nf), dtype=dt, device=dev)
            norm = torch.empty((ntasks,), dtype=torch.float64, device=dev)
            lipschitz = torch.empty((ntasks,), dtype=torch.float64, device=dev)
            self.backend.power_init(v, seed)
            for _ in range(n_power):
                P = self.backend.reduced_partial(self.X_local, v, None, self.group)
                self.backend.power_step(P, v, norm, lipschitz, lambda2)
            beta = torch.zeros((ntasks, nt, nf), dtype=dt, device=dev)
        for it in range(start, n_iter):
            P = self.backend.reduced_partial(self.X_local, beta, self.Y_local, self.group)
            self.backend.prox_update(P, beta, lipschitz, lambda1, lambda2)
            if checkpoint is not None:
                checkpoint(it + 1, beta, lipschitz)
        return beta, lipschitz
