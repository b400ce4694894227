"""Streaming (host chunks, accumulated statistics) and the sharded step on one
GPU, checked against a single E-step call and the oracle."""

import numpy as np
import pytest
import torch

import gmm_data
import gmm_stream as GS
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu


def test_stream_estep_matches_single_call():
    X, mu, lss, lpi = gmm_data.make_config("c2", N=60_000)
    chunks = [X[i:i + 17_000].pin_memory() for i in range(0, X.shape[0], 17_000)]
    logZ, Nk, mu_acc, sig = GS.stream_estep(chunks, mu, lss, lpi, keep_logZ=True)
    torch.cuda.synchronize()
    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    assert_parity(tuple(t.cpu().numpy() for t in (logZ, Nk, mu_acc, sig)), ref,
                  what="stream_estep")


def test_sharded_step_single_rank_and_generator():
    dev = torch.device("cuda")
    centres = GS.mixture_centres(64, 32, 5, dev)
    X = GS.generate_rows(0, 20_000, centres, 5)
    # row-keyed: a shifted window sees the same rows
    X2 = GS.generate_rows(5_000, 10_000, centres, 5)
    torch.cuda.synchronize()
    assert torch.equal(X[5_000:15_000], X2)
    ids = GS.pick_mean_rows(20_000, 64, 5)
    mu = GS.generate_row_ids(ids.to(dev), centres, 5)
    assert torch.equal(mu, X[ids.to(dev)])
    lss = torch.zeros(64, device=dev)
    lpi = torch.full((64,), -np.log(64.0), device=dev)
    out = GS.ShardedEStep("iso")(X, mu, lss, lpi)
    torch.cuda.synchronize()
    ref = O.estep_iso(X.cpu().numpy(), mu.cpu().numpy(), lss.cpu().numpy(), lpi.cpu().numpy())
    assert_parity(tuple(t.cpu().numpy() for t in out), ref, what="sharded step, 1 rank")
