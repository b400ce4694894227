"""N>1 host logic on CPU ranks (gloo, world_size 2): row sharding, the packed
[Nk | mu_acc | sig] buffer and its single all-reduce, and failure detection
(a rank that leaves makes the other's collective fail instead of hanging).

The per-rank E-step here is the CPU oracle injected through ``estep_fn``;
the product path calls the CUDA library and has no CPU fallback."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_estep(variant):
    def run(X, mu, cov, lpi, out):
        from oracle import gmm_oracle as O
        fn = {"iso": O.estep_iso, "diag": O.estep_diag, "full": O.estep_full}[variant]
        res = fn(X.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
        for t, r in zip(out, res):
            t.copy_(torch.from_numpy(np.asarray(r, dtype=np.float32)).reshape(t.shape))
        return out
    return run


def _data(variant, N=1003, K=7, D=5):
    g = torch.Generator().manual_seed(11)
    X = torch.randn(N, D, generator=g)
    mu = torch.randn(K, D, generator=g)
    cov = {"iso": 0.2 * torch.randn(K, generator=g),
           "diag": 0.2 * torch.randn(K, D, generator=g),
           "full": torch.tril(0.1 * torch.randn(K, D, D, generator=g), -1) + torch.eye(D)}[variant]
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, cov, lpi


def _worker(rank, world, port, variant, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "flash-gmm_b200")]
    import datetime
    import torch.distributed as dist
    import gmm_stream as GS
    from oracle import gmm_oracle as O
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=20))
        X, mu, cov, lpi = _data(variant)
        lo, hi = GS.shard_rows(X.shape[0], rank, world)
        step = GS.ShardedEStep(variant, estep_fn=_cpu_estep(variant))
        logZ, Nk, mu_acc, sig = step(X[lo:hi], mu, cov, lpi)
        fn = {"iso": O.estep_iso, "diag": O.estep_diag, "full": O.estep_full}[variant]
        ref = fn(X.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
        err = [float(np.max(np.abs(logZ.numpy() - ref[0][lo:hi])))]
        for a, b in zip((Nk, mu_acc, sig), ref[1:]):
            err.append(float(np.max(np.abs(a.numpy() - b)) / np.max(np.abs(b))))
        q.put((rank, err, hi - lo))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), -1))


@pytest.mark.parametrize("variant", ["iso", "diag", "full"])
def test_sharded_estep_two_ranks(variant):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, variant, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    rows = 0
    for rank, err, n in sorted(res):
        assert n > 0, err
        rows += n
        assert err[0] < 1e-4 and max(err[1:]) < 1e-5, (rank, err)
    assert rows == 1003


def _leaver(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "flash-gmm_b200")]
    import datetime
    import torch.distributed as dist
    import gmm_stream as GS
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((1, "left"))
        q.close()
        q.join_thread()  # flush the message before leaving
        os._exit(0)  # leaves between steps, no collective in flight
    X, mu, cov, lpi = _data("iso")
    step = GS.ShardedEStep("iso", estep_fn=_cpu_estep("iso"))
    try:
        step(X, mu, cov, lpi)
        q.put((0, "no error"))
    except Exception as e:
        q.put((0, "raised " + type(e).__name__))


def test_rank_leaving_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("raised"), res[0]


def test_shard_rows_partition():
    import gmm_stream as GS
    for N in (0, 1, 7, 1000, 1003):
        for w in (1, 2, 3, 8):
            spans = [GS.shard_rows(N, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
