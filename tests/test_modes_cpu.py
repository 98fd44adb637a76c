"""Host-side rules of the 'factored' state precision and of spectral
normalisation, on CPU tensors (no kernels run):

  * the sign array lives in storage that is a whole number of 4-byte words
    (the kernel sets sign bits with 32-bit atomics), including after a
    checkpoint written elsewhere is loaded (`ensure_sign_words`);
  * scale_update's choice per param (scaled_optm.py:54-72, 108-116): max-abs
    scaling for 1-D params and DoRA magnitudes, spectral scaling for params of
    two or more dims, refused for OFT blocks and for 2-D params the reference
    gives no singular vectors;
  * init_spectral_norm's shapes and unit norms (scaled_optm.py:118-142).
"""
import numpy as np
import pytest
import torch

from advanced_optimizers_b200.optim._adam_family import (
    SpectralInit, ensure_sign_words, init_adam_state, is_spectral, sign_storage, spectral_kind)


@pytest.mark.parametrize("d1,pd2", [(63, 5), (40, 5), (1, 1), (7, 3), (64, 4)])
def test_sign_storage_is_whole_words(d1, pd2):
    s = sign_storage(d1, pd2, torch.device("cpu"))
    assert s.shape == (d1, pd2) and s.dtype == torch.uint8 and s.is_contiguous()
    n = d1 * pd2
    assert s.untyped_storage().nbytes() - s.storage_offset() >= ((n + 3) // 4) * 4
    assert s.data_ptr() % 4 == 0
    assert int(s.sum()) == 0


def test_loaded_sign_array_is_rehomed_with_its_values():
    # a (63, 5) array as another library would save it: 315 bytes, no padding
    g = torch.Generator().manual_seed(0)
    loaded = torch.randint(0, 256, (63, 5), generator=g, dtype=torch.uint8)
    loaded = loaded.clone()                      # storage of exactly 315 bytes
    assert loaded.untyped_storage().nbytes() == 315
    st = {"sign": loaded}
    ensure_sign_words(st)
    assert st["sign"] is not loaded
    assert torch.equal(st["sign"], loaded)
    assert st["sign"].untyped_storage().nbytes() >= 316
    # an array that already ends on a word is kept as it is
    ok = sign_storage(10, 4, torch.device("cpu"))
    st = {"sign": ok}
    ensure_sign_words(st)
    assert st["sign"] is ok


def test_factored_state_layout_matches_the_reference_keys():
    p = torch.zeros(300, 70, dtype=torch.bfloat16)
    st = {}
    init_adam_state(p, st, precision="factored", factored_2nd=False, beta1=0.9, vector_reshape=False,
                    centered_wd=0.0, centered_wd_mode="float8", fisher_wd=False)
    assert st["factored"] is True and st["effective_shape"] == (150, 140)
    assert st["mu_m_nmf"].shape == (150,) and st["mv_m_nmf"].shape == (140,)
    assert st["sign"].shape == (150, 18) and st["sign"].dtype == torch.uint8
    assert st["mu_v_nmf"].dtype == torch.float32 and st["mv_v_nmf"].shape == (140,)
    assert st["shifter"].tolist() == [1, 2, 4, 8, 16, 32, 64, 128]
    # a 1-D param of a 'factored' group keeps float32 m and v
    v = torch.zeros(96, dtype=torch.bfloat16)
    sv = {}
    init_adam_state(v, sv, precision="factored", factored_2nd=False, beta1=0.9, vector_reshape=False,
                    centered_wd=0.0, centered_wd_mode="float8", fisher_wd=False)
    assert sv["factored"] is False
    assert sv["exp_avg"].dtype == torch.float32 and sv["exp_avg_sq"].dtype == torch.float32
    # without momentum only the rank-1 v exists
    s0 = {}
    init_adam_state(p, s0, precision="factored", factored_2nd=False, beta1=0.0, vector_reshape=False,
                    centered_wd=0.0, centered_wd_mode="float8", fisher_wd=False)
    assert "sign" not in s0 and "mu_m_nmf" not in s0 and "mu_v_nmf" in s0


def _marked(shape, **attrs):
    p = torch.nn.Parameter(torch.zeros(shape))
    for k, v in attrs.items():
        setattr(p, k, v)
    return p


def test_spectral_kind_follows_scale_update():
    assert spectral_kind(_marked((64,))) == "maxabs"
    assert spectral_kind(_marked((64, 32))) == "spectral"
    assert spectral_kind(_marked((8, 4, 3))) == "spectral"
    assert spectral_kind(_marked((64, 32), _is_dora_scale=True)) == "maxabs"
    with pytest.raises(NotImplementedError):
        spectral_kind(_marked((4, 6), _is_oft=True))
    with pytest.raises(NotImplementedError):
        spectral_kind(_marked((64, 32), is_hidden=False))
    with pytest.raises(NotImplementedError):
        spectral_kind(_marked((64, 32), is_vector=True))
    assert is_spectral(_marked((64, 32))) and not is_spectral(_marked((64,)))


def test_spectral_init_shapes_and_unit_norms():
    init = SpectralInit(seed=7)
    p = _marked((12, 5, 2))                 # d_out 12, d_in 10
    st = {}
    init(st, p)
    assert st["spectral_u"].shape == (12,) and st["spectral_v"].shape == (10,)
    assert st["spectral_u"].dtype == p.dtype
    for k in ("spectral_u", "spectral_v"):
        assert abs(float(st[k].norm()) - 1.0) < 1e-5
    # a 1-D param gets no singular vectors (its update is max-abs scaled)
    s1 = {}
    init(s1, _marked((12,)))
    assert "spectral_u" not in s1
    # the draws are reproducible for a given seed
    st2 = {}
    SpectralInit(seed=7)(st2, p)
    assert np.array_equal(st["spectral_v"].numpy(), st2["spectral_v"].numpy())
