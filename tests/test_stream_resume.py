"""Resumable streamed E-step (gmm_stream.resumable_stream_estep): checkpoint
state (next_row, Nk, mu_acc, sig, sum logZ), resume after a stop, refusal of
a state made for another pass.

CPU tests drive the host logic with a window function built on the fp64
oracle (summing each chunk's statistics into the running fp32 state, as the
library's accumulate flag does); the GPU test runs the library's
stream_estep and checks that a pass stopped and resumed ends with the same
bits as an uninterrupted one.
"""

import numpy as np
import pytest
import torch

import gmm_data
import gmm_stream as GS
from oracle import gmm_oracle as O
from parity import assert_parity


class Stop(Exception):
    pass


def _reader(X, stop_at_row=None):
    def read(row0, n):
        if stop_at_row is not None and row0 >= stop_at_row:
            raise Stop(row0)
        return X[row0:row0 + n].clone()
    return read


def _oracle_window(chunks, mu, cov, lpi, init):
    """CPU stand-in for stream_estep(init=...): per chunk, statistics in fp64
    added to the running fp32 accumulators in chunk order."""
    Nk, mu_acc, sig = (t.clone().float() for t in init)
    logZ = []
    for c in chunks:
        lz, nk, ma, sg = O.estep_iso(c.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
        Nk += torch.from_numpy(nk).float()
        mu_acc += torch.from_numpy(ma).float()
        sig += torch.from_numpy(sg).float()
        logZ.append(torch.from_numpy(lz).float())
    return torch.cat(logZ), Nk, mu_acc, sig


def _case(N=5_000, K=40, D=12):
    return gmm_data.iso_mixture(N, K, D, seed=7)


def test_resume_after_stop_matches_uninterrupted_pass(tmp_path):
    X, mu, lss, lpi = _case()
    N = X.shape[0]
    kw = dict(variant="iso", chunk_rows=700, checkpoint_every=2, window_fn=_oracle_window)
    full = GS.resumable_stream_estep(_reader(X), N, mu, lss, lpi, **kw)
    assert full.done and full.next_row == N

    ck = str(tmp_path / "estep.ckpt")
    with pytest.raises(Stop):
        GS.resumable_stream_estep(_reader(X, stop_at_row=3 * 1400), N, mu, lss, lpi,
                                  checkpoint_path=ck, **kw)
    saved = GS.StreamState.load(ck)
    assert saved.next_row == 3 * 1400 and not saved.done  # last completed window
    sink = {}
    resumed = GS.resumable_stream_estep(_reader(X), N, mu, lss, lpi, checkpoint_path=ck,
                                        logz_sink=lambda r, z: sink.__setitem__(r, z), **kw)
    for a, b in ((full.Nk, resumed.Nk), (full.mu_acc, resumed.mu_acc), (full.sig, resumed.sig)):
        assert torch.equal(a, b)
    assert resumed.sum_logZ == pytest.approx(full.sum_logZ, rel=1e-12)
    assert min(sink) == 3 * 1400 and GS.StreamState.load(ck).done

    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    assert_parity((ref[0], resumed.Nk.numpy(), resumed.mu_acc.numpy(), resumed.sig.numpy()),
                  ref, what="resumed streamed pass vs one oracle pass")
    assert resumed.sum_logZ == pytest.approx(float(np.sum(ref[0], dtype=np.float64)), rel=1e-6)


def test_state_for_another_pass_is_refused(tmp_path):
    X, mu, lss, lpi = _case(N=1_000)
    ck = str(tmp_path / "s.ckpt")
    GS.StreamState.start("iso", 1_000, 300, 40, 12).save(ck)
    with pytest.raises(ValueError, match="another pass"):
        GS.resumable_stream_estep(_reader(X), 1_000, mu, lss, lpi, chunk_rows=250,
                                  checkpoint_path=ck, window_fn=_oracle_window)
    st = GS.StreamState.start("iso", 1_000, 300, 40, 12)
    st.next_row = 450
    with pytest.raises(ValueError, match="chunk boundary"):
        GS.resumable_stream_estep(_reader(X), 1_000, mu, lss, lpi, chunk_rows=300, state=st,
                                  window_fn=_oracle_window)


def test_finished_state_and_empty_pass(tmp_path):
    X, mu, lss, lpi = _case(N=600)
    st = GS.resumable_stream_estep(_reader(X), 0, mu, lss, lpi, chunk_rows=256,
                                   window_fn=_oracle_window)
    assert st.done and float(st.Nk.sum()) == 0.0 and st.sum_logZ == 0.0
    ck = str(tmp_path / "f.ckpt")
    a = GS.resumable_stream_estep(_reader(X), 600, mu, lss, lpi, chunk_rows=256,
                                  checkpoint_path=ck, window_fn=_oracle_window)
    # a finished checkpoint resumes to itself without reading rows
    b = GS.resumable_stream_estep(_reader(X, stop_at_row=0), 600, mu, lss, lpi, chunk_rows=256,
                                  checkpoint_path=ck, window_fn=_oracle_window)
    assert torch.equal(a.Nk, b.Nk) and b.sum_logZ == a.sum_logZ


@pytest.mark.gpu
def test_gpu_resume_is_bitwise_and_matches_one_call(tmp_path):
    import _fgmm_lib as L
    X, mu, lss, lpi = gmm_data.make_config("c2", N=90_000)
    Xh = X.pin_memory()
    dev = torch.device("cuda")
    mud, lssd, lpid = mu.to(dev), lss.to(dev), lpi.to(dev)
    N = X.shape[0]

    def read(stop=None):
        def f(row0, n):
            if stop is not None and row0 >= stop:
                raise Stop(row0)
            return Xh[row0:row0 + n]
        return f

    kw = dict(variant="iso", chunk_rows=16_384, checkpoint_every=2)
    full = GS.resumable_stream_estep(read(), N, mud, lssd, lpid, **kw)
    ck = str(tmp_path / "g.ckpt")
    with pytest.raises(Stop):
        GS.resumable_stream_estep(read(stop=2 * 32_768), N, mud, lssd, lpid,
                                  checkpoint_path=ck, **kw)
    resumed = GS.resumable_stream_estep(read(), N, mud, lssd, lpid, checkpoint_path=ck, **kw)
    for a, b in ((full.Nk, resumed.Nk), (full.mu_acc, resumed.mu_acc), (full.sig, resumed.sig)):
        assert torch.equal(a, b)
    one = L.estep(L.FGMM_VARIANT_ISO, X.to(dev), mud, lssd, lpid)
    torch.cuda.synchronize()
    assert_parity((one[0].cpu().numpy(), resumed.Nk.numpy(), resumed.mu_acc.numpy(),
                   resumed.sig.numpy()), tuple(t.cpu().numpy() for t in one),
                  what="resumed stream vs one call")
    assert resumed.sum_logZ == pytest.approx(float(one[0].double().sum()), rel=1e-6)
