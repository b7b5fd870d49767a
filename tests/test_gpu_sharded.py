"""Observation-sharded gradient and fit across 2 GPUs (NCCL), one process
per GPU, checked against the single-GPU entry points on the full data.
Skipped when fewer than two GPUs are visible."""
import os
import socket
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs two CUDA devices", allow_module_level=True)

import torch.multiprocessing as mp  # noqa: E402


def _problem(dt):
    rng = np.random.default_rng(8)
    nobs, ntasks, nf, nt = 200_003, 2, 96, 2
    X = rng.uniform(-1, 1, (nobs, ntasks, nf)).astype(dt)
    bt = rng.normal(size=(ntasks, nt, nf)) * (rng.uniform(size=(ntasks, nt, nf)) < 0.3)
    Y = (np.einsum("otf,tkf->otk", X.astype(np.float64), bt) + 0.1 * rng.normal(size=(nobs, ntasks, nt))).astype(dt)
    M = rng.uniform(0, 1, (ntasks, nt, nf)).astype(dt)
    return X, Y, M


def _worker(rank, world, port, outdir, dt_name, exchange):
    import torch.distributed as dist
    from datetime import timedelta

    from gpu_algos_b200.sharded import CudaBackend, PeerBackend, PeerGroup, ShardedGLM, obs_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        X, Y, M = _problem(np.dtype(dt_name))
        lo, hi = obs_range(X.shape[0], world, rank)
        peer = PeerGroup(max_elems=M.size, timeout_ms=5000.0) if exchange == "peer" else None
        backend = PeerBackend(peer) if peer is not None else CudaBackend()
        sh = ShardedGLM(torch.from_numpy(X[lo:hi].copy()).cuda(), torch.from_numpy(Y[lo:hi].copy()).cuda(),
                        backend)
        g = sh.gradient(torch.from_numpy(M).cuda(), 0.2, 0.3)
        beta, lip = sh.fit_elastic_net(50.0, 5.0, n_power=20, n_iter=40, seed=11)
        torch.cuda.synchronize()
        if peer is not None:
            assert peer.status() == 0
            peer.close()
        np.save(os.path.join(outdir, f"g{rank}.npy"), g.cpu().numpy())
        np.save(os.path.join(outdir, f"b{rank}.npy"), beta.cpu().numpy())
        np.save(os.path.join(outdir, f"l{rank}.npy"), lip.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_two_gpu_sharded_matches_single_gpu(dt, exchange):
    outdir = tempfile.mkdtemp()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, outdir, np.dtype(dt).name, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive(), "a rank hung"
        assert p.exitcode == 0
    from gpu_algos_b200 import glm

    X, Y, M = _problem(dt)
    tX, tY, tM = (torch.from_numpy(a).cuda() for a in (X, Y, M))
    g_ref = glm.gradient(tX, tM, tY, 0.2, 0.3).cpu().numpy()
    b_ref, l_ref = glm.fit_elastic_net(tX, tY, 50.0, 5.0, n_power=20, n_iter=40, seed=11)
    b_ref, l_ref = b_ref.cpu().numpy(), l_ref.cpu().numpy()
    g0, g1 = np.load(os.path.join(outdir, "g0.npy")), np.load(os.path.join(outdir, "g1.npy"))
    assert np.array_equal(g0, g1)
    tol = 1e-4 if dt == np.float32 else 1e-11
    assert np.max(np.abs(g0 - g_ref) / np.abs(g_ref)) <= tol
    b0 = np.load(os.path.join(outdir, "b0.npy"))
    assert np.array_equal(b0, np.load(os.path.join(outdir, "b1.npy")))
    assert np.allclose(np.load(os.path.join(outdir, "l0.npy")), l_ref, rtol=tol)
    assert np.max(np.abs(b0 - b_ref)) <= (1e-3 if dt == np.float32 else 1e-9) * np.max(np.abs(b_ref))


def _wide_problem(dt):
    """Many targets: float32 takes the dense tensor-core path, float64 the tiles path."""
    rng = np.random.default_rng(9)
    nobs, ntasks, nf, nt = 60_001, 2, 128 if dt == np.float32 else 64, 40 if dt == np.float32 else 16
    X = rng.uniform(-1, 1, (nobs, ntasks, nf)).astype(dt)
    Y = rng.normal(size=(nobs, ntasks, nt)).astype(dt)
    M = rng.normal(size=(ntasks, nt, nf)).astype(dt)
    return X, Y, M


def _worker_wide(rank, world, port, outdir, dt_name, exchange):
    import torch.distributed as dist
    from datetime import timedelta

    from gpu_algos_b200 import capi
    from gpu_algos_b200.sharded import CudaBackend, PeerBackend, PeerGroup, ShardedGLM, obs_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        X, Y, M = _wide_problem(np.dtype(dt_name))
        lo, hi = obs_range(X.shape[0], world, rank)
        peer = PeerGroup(max_elems=M.size, timeout_ms=5000.0) if exchange == "peer" else None
        backend = PeerBackend(peer) if peer is not None else CudaBackend()
        sh = ShardedGLM(torch.from_numpy(X[lo:hi].copy()).cuda(), torch.from_numpy(Y[lo:hi].copy()).cuda(),
                        backend)
        g = sh.gradient(torch.from_numpy(M).cuda(), 0.2, 0.3)
        torch.cuda.synchronize()
        path = capi.last_path()
        if peer is not None:
            assert peer.status() == 0
            peer.close()
        np.save(os.path.join(outdir, f"g{rank}.npy"), g.cpu().numpy())
        with open(os.path.join(outdir, f"path{rank}.txt"), "w") as f:
            f.write(path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_two_gpu_sharded_dense_and_tiles_paths(dt, exchange):
    outdir = tempfile.mkdtemp()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker_wide, args=(r, 2, port, outdir, np.dtype(dt).name, exchange))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive(), "a rank hung"
        assert p.exitcode == 0
    from gpu_algos_b200 import glm

    for r in range(2):
        with open(os.path.join(outdir, f"path{r}.txt")) as f:
            assert f.read() == ("dense" if dt == np.float32 else "tiles")
    X, Y, M = _wide_problem(dt)
    tX, tY, tM = (torch.from_numpy(a).cuda() for a in (X, Y, M))
    g_ref = glm.gradient(tX, tM, tY, 0.2, 0.3).cpu().numpy()
    g0, g1 = np.load(os.path.join(outdir, "g0.npy")), np.load(os.path.join(outdir, "g1.npy"))
    assert np.array_equal(g0, g1)
    floor = 1e-3 * np.abs(g_ref).max()
    tol = 1e-4 if dt == np.float32 else 1e-11
    assert np.max(np.abs(g0 - g_ref) / np.maximum(np.abs(g_ref), floor)) <= tol


def _problem16():
    """_problem's data scaled by 0.1: the gradient's largest element (about
    4e3) stays inside half's range (65504)."""
    X, Y, M = _problem(np.float32)
    return X * np.float32(0.1), Y * np.float32(0.1), M


def _worker16(rank, world, port, outdir, dt_name, exchange):
    import torch.distributed as dist
    from datetime import timedelta

    from gpu_algos_b200.sharded import CudaBackend, PeerBackend, PeerGroup, ShardedGLM, obs_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        X, Y, M = _problem16()
        dt = getattr(torch, dt_name)
        lo, hi = obs_range(X.shape[0], world, rank)
        peer = PeerGroup(max_elems=M.size, timeout_ms=5000.0) if exchange == "peer" else None
        backend = PeerBackend(peer) if peer is not None else CudaBackend()
        sh = ShardedGLM(torch.from_numpy(X[lo:hi].copy()).cuda().to(dt), torch.from_numpy(Y[lo:hi].copy()).cuda().to(dt),
                        backend)
        g = sh.gradient(torch.from_numpy(M).cuda().to(dt), 0.2, 0.3)
        torch.cuda.synchronize()
        if peer is not None:
            assert peer.status() == 0
            peer.close()
        np.save(os.path.join(outdir, f"g{rank}.npy"), g.float().cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("dt_name", ["float16", "bfloat16"])
def test_two_gpu_sharded_16bit_gradient(dt_name, exchange):
    """half and bfloat16: glmb_gradient_partial/finalize (NCCL) and
    glmb_gradient_sharded (peer exchange) on two GPUs give identical bits on
    both ranks and match the one-GPU gradient of the full data to one unit in
    the last place of the type (2^-10 half, 2^-7 bfloat16, relative; floor
    1e-2 of the largest element): the partial sums are exact to float
    precision either way, and each result is rounded once."""
    outdir = tempfile.mkdtemp()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker16, args=(r, 2, port, outdir, dt_name, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive(), "a rank hung"
        assert p.exitcode == 0
    from gpu_algos_b200 import glm

    dt = getattr(torch, dt_name)
    X, Y, M = _problem16()
    tX, tY, tM = (torch.from_numpy(a).cuda().to(dt) for a in (X, Y, M))
    g_ref = glm.gradient(tX, tM, tY, 0.2, 0.3).float().cpu().numpy().astype(np.float64)
    g0, g1 = np.load(os.path.join(outdir, "g0.npy")), np.load(os.path.join(outdir, "g1.npy"))
    assert np.array_equal(g0, g1)
    assert np.isfinite(g_ref).all()
    tol = 2.0 ** -10 if dt_name == "float16" else 2.0 ** -7
    den = np.maximum(np.abs(g_ref), 1e-2 * np.abs(g_ref).max())
    assert np.max(np.abs(g0 - g_ref) / den) <= tol
