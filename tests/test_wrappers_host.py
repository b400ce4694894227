"""Host-side behaviour of the drop-in entry points that needs no GPU: the
reference's assertion types and messages (flash_gmm.py:189-190,
flash_gmm_diag_h100.py:313-315, flash_gmm_full_h100.py:264-266)."""

import pytest
import torch

import flash_gmm
import flash_gmm_diag_h100
import flash_gmm_full_h100
import flash_gmm_h100


def test_block_d_assert_message():
    X, mu = torch.zeros(4, 200), torch.zeros(3, 200)
    with pytest.raises(AssertionError, match=r"D=200 exceeds BLOCK_D=128; increase BLOCK_D\."):
        flash_gmm.flash_gmm_estep(X, mu, torch.zeros(3), torch.zeros(3))


def test_cpu_inputs_rejected():
    X, mu = torch.zeros(4, 8), torch.zeros(3, 8)
    with pytest.raises(AssertionError, match="Inputs must be on GPU."):
        flash_gmm.flash_gmm_estep(X, mu, torch.zeros(3), torch.zeros(3))
    with pytest.raises(AssertionError):
        flash_gmm_h100.flash_gmm_estep(X, mu, torch.zeros(3), torch.zeros(3))


def test_diag_shape_assert():
    X, mu = torch.zeros(4, 8), torch.zeros(3, 8)
    with pytest.raises(AssertionError, match=r"log_sigma_sq must be \(K, D\)=\(3, 8\), got \(3,\)"):
        flash_gmm_diag_h100.flash_gmm_estep_diag(X, mu, torch.zeros(3), torch.zeros(3))


def test_full_shape_assert():
    X, mu = torch.zeros(4, 8), torch.zeros(3, 8)
    with pytest.raises(AssertionError,
                       match=r"prec_chol must be \(K, D, D\)=\(3, 8, 8\), got \(3, 8\)"):
        flash_gmm_full_h100.flash_gmm_estep_full(X, mu, torch.zeros(3, 8), torch.zeros(3))


def test_missing_library_raises_instead_of_falling_back(monkeypatch, tmp_path):
    """Without the built library the binding raises: there is no CPU path."""
    import _fgmm_lib as L
    monkeypatch.setattr(L, "_lib", None)
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "libflashgmm_sm100.so"))
    with pytest.raises(RuntimeError, match="no fallback implementation"):
        L.load()
    with pytest.raises(RuntimeError, match="no fallback implementation"):
        L.workspace_bytes(L.FGMM_VARIANT_ISO, 10, 4, 8)
