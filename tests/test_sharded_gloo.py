"""Host-side logic of the observation-sharded path on CPU ranks (gloo,
world size 2): the shard split, the single all-reduce per evaluation, the
fit loop, checkpoint/resume, and failure detection of a rank that dies.

The per-rank arithmetic comes from a NumPy backend built on the oracle (the
CUDA backend is exercised by the GPU tests and bench.py); what is under test
here is the orchestration in gpu_algos_b200/sharded.py.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gpu_algos_b200.sharded import POWER_SAFETY, Backend, ShardedGLM, obs_range, task_range


class OracleBackend(Backend):
    """Float64 per-rank arithmetic on the CPU, from the oracle."""

    def __init__(self):
        from oracle import pyoracle

        self.o = pyoracle

    def partial(self, X, M, Y):
        g = self.o.gradient(X.numpy(), M.numpy(), None if Y is None else Y.numpy(), with_reg=False)
        return torch.from_numpy(g / 2.0)

    def finalize(self, P, M, lam, alpha, out):
        Mn = M.numpy()
        g = 2 * P.numpy() + lam * (alpha * np.sign(Mn) + 2 * (1 - alpha) * Mn)
        out.copy_(torch.from_numpy(g))
        return out

    def power_init(self, v, seed):
        ntasks, _, nf = v.shape
        v0 = self.o.power_start(ntasks * nf, seed).reshape(ntasks, 1, nf)
        v0 /= np.linalg.norm(v0, axis=2, keepdims=True)
        v.copy_(torch.from_numpy(v0))
        return v

    def power_step(self, P, v, norm, lipschitz, lambda2):
        g = 2 * P.numpy()
        n = np.linalg.norm(g, axis=(1, 2))
        v.copy_(torch.from_numpy(g / n[:, None, None]))
        norm.copy_(torch.from_numpy(n))
        lipschitz.copy_(torch.from_numpy(POWER_SAFETY * n + 2 * lambda2))
        return v

    def prox_update(self, P, beta, lipschitz, lambda1, lambda2):
        b = beta.numpy()
        L = lipschitz.numpy()[:, None, None]
        z = b - (2 * P.numpy() + 2 * lambda2 * b) / L
        beta.copy_(torch.from_numpy(np.sign(z) * np.maximum(np.abs(z) - lambda1 / L, 0)))
        return beta


def _problem():
    rng = np.random.default_rng(21)
    nobs, ntasks, nf, nt = 1001, 2, 7, 3
    X = rng.normal(size=(nobs, ntasks, nf))
    bt = rng.normal(size=(ntasks, nt, nf)) * (rng.uniform(size=(ntasks, nt, nf)) < 0.5)
    Y = np.einsum("otf,tkf->otk", X, bt) + 0.1 * rng.normal(size=(nobs, ntasks, nt))
    M = rng.normal(size=(ntasks, nt, nf))
    return X, Y, M


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir, mode):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        X, Y, M = _problem()
        lo, hi = obs_range(X.shape[0], world, rank)
        sh = ShardedGLM(torch.from_numpy(X[lo:hi].copy()), torch.from_numpy(Y[lo:hi].copy()), OracleBackend())
        if mode == "gradient":
            g = sh.gradient(torch.from_numpy(M), 0.3, 0.4)
            np.save(os.path.join(outdir, f"grad{rank}.npy"), g.numpy())
        elif mode == "fit":
            beta, lip = sh.fit_elastic_net(20.0, 3.0, n_power=30, n_iter=60, seed=5)
            np.save(os.path.join(outdir, f"beta{rank}.npy"), beta.numpy())
            np.save(os.path.join(outdir, f"lip{rank}.npy"), lip.numpy())
        elif mode == "resume":
            snaps = {}

            def ck(it, beta, lip):
                if it == 25:
                    snaps["s"] = (it, beta.clone(), lip.clone())

            full, _ = sh.fit_elastic_net(20.0, 3.0, n_power=30, n_iter=60, seed=5, checkpoint=ck)
            again, _ = sh.fit_elastic_net(20.0, 3.0, n_power=30, n_iter=60, seed=5, resume=snaps["s"])
            np.save(os.path.join(outdir, f"resume{rank}.npy"), np.stack([full.numpy(), again.numpy()]))
        elif mode == "rank_dies":
            if rank == 1:
                raise SystemExit(3)  # leaves between steps, before the collective
            try:
                sh.gradient(torch.from_numpy(M), 0.3, 0.4)
                np.save(os.path.join(outdir, "no_error.npy"), np.zeros(1))
            except Exception as e:  # gloo reports the lost peer or the timeout
                with open(os.path.join(outdir, "error.txt"), "w") as f:
                    f.write(type(e).__name__ + ": " + str(e)[:200])
    finally:
        if mode != "rank_dies":
            dist.destroy_process_group()


def _spawn(mode, world=2):
    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, outdir, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail(f"{mode}: a rank hung")
    return outdir, [p.exitcode for p in procs]


def test_obs_and_task_ranges():
    for nobs in (0, 1, 7, 1000, 1001):
        for world in (1, 2, 3, 8):
            blocks = [obs_range(nobs, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == nobs
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in blocks]
            assert max(sizes) - min(sizes) <= 1
    assert task_range(64, 8, 3) == (24, 32)
    with pytest.raises(ValueError):
        obs_range(10, 2, 2)


def test_sharded_gradient_matches_single_process(oracle):
    outdir, codes = _spawn("gradient")
    assert codes == [0, 0]
    g0, g1 = (np.load(os.path.join(outdir, f"grad{r}.npy")) for r in range(2))
    assert np.array_equal(g0, g1)  # every rank ends with the same bits
    X, Y, M = _problem()
    ref = oracle.gradient(X, M, Y, 0.3, 0.4, True)
    assert np.allclose(g0, ref, rtol=1e-12, atol=1e-9)


def test_sharded_fit_matches_oracle_fit(oracle):
    outdir, codes = _spawn("fit")
    assert codes == [0, 0]
    b0, b1 = (np.load(os.path.join(outdir, f"beta{r}.npy")) for r in range(2))
    assert np.array_equal(b0, b1)
    X, Y, _ = _problem()
    ntasks, nf = X.shape[1], X.shape[2]
    ob, olip = oracle.fit(X, Y, 20.0, 3.0, oracle.power_start(ntasks * nf, 5), n_power=30, n_iter=60)
    assert np.allclose(np.load(os.path.join(outdir, "lip0.npy")), olip, rtol=1e-10)
    assert np.allclose(b0, ob, rtol=1e-9, atol=1e-12)


def test_checkpoint_resume_is_exact():
    outdir, codes = _spawn("resume")
    assert codes == [0, 0]
    for r in range(2):
        full, again = np.load(os.path.join(outdir, f"resume{r}.npy"))
        assert np.array_equal(full, again)


def test_dead_rank_is_detected_not_hung():
    outdir, codes = _spawn("rank_dies")
    assert codes[1] == 3
    assert os.path.exists(os.path.join(outdir, "error.txt")), "the surviving rank did not see the failure"
    assert not os.path.exists(os.path.join(outdir, "no_error.npy"))
