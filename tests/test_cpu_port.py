"""The fp32 torch-CPU ports that bench.py times as the CPU baseline (and as the
reference arm) compute the same E-step as the fp64 oracle, to the parity bar,
on every fixture of the reference's own outputs and on small scaled benchmark
configurations (several row chunks, -inf weights included)."""

import numpy as np
import pytest
import torch

import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity, golden_inputs, golden_names, load_golden, variant_of

PORT = {"iso": O.estep_iso_cpu_fp32, "diag": O.estep_diag_cpu_fp32,
        "full": O.estep_full_cpu_fp32}
ORACLE = {"iso": O.estep_iso, "diag": O.estep_diag, "full": O.estep_full}
NAMES = [n for n in golden_names() if n != "diag_slab_overlap_defect"]


def _port(variant, X, mu, cov, lpi, **kw):
    t = [torch.as_tensor(np.asarray(a)) for a in (X, mu, cov, lpi)]
    return [o.double().numpy() for o in PORT[variant](*t, **kw)]


@pytest.mark.parametrize("name", NAMES)
def test_port_matches_oracle_on_fixture_inputs(name):
    z = load_golden(name)
    X, mu, cov, lpi = golden_inputs(name, z)
    v = variant_of(name)
    assert_parity(_port(v, X, mu, cov, lpi), ORACLE[v](X, mu, cov, lpi), what=name)


@pytest.mark.parametrize("cfg,N", [("c2", 5000), ("c3", 5000), ("c4", 3000)])
def test_port_matches_oracle_scaled_configs(cfg, N):
    X, mu, cov, lpi = gmm_data.make_config(cfg, N=N)
    lpi = lpi.clone()
    lpi[3] = float("-inf")                        # a component with zero weight
    v = gmm_data.CONFIGS[cfg]["kind"]
    ref = ORACLE[v](X.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
    # chunks smaller than N: the per-chunk accumulation is exercised
    out = _port(v, X, mu, cov, lpi, chunk=1024)
    assert_parity(out, ref, what=f"{cfg} port")
    assert np.all(out[1][3] == 0.0)
