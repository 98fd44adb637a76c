"""The stochastic-rounding noise generator and the unbiasedness of the
stochastic roundings under it (GPU).

  * Philox4x32-10 known-answer vectors (Salmon et al., SC'11, Random123) and
    agreement with a Python restatement of the algorithm on random inputs;
  * advopt_noise_fill reproduces the counter mapping the kernels use and is
    uniform over [0, 65536) (chi-square over 256 buckets);
  * bf16 stochastic rounding of an AdamW step over 2^20 equal elements rounds
    up with the probability the exact fp32 result implies (5 sigma);
  * int8 stochastic quantisation of the momentum is unbiased: the mean of
    code * scale - m over 2^20 elements is within 5 sigma of zero."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox_py(c, k):
    c = list(c)
    k0, k1 = k
    for _ in range(10):
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & MASK, p1 & MASK, ((p0 >> 32) ^ c[3] ^ k1) & MASK, p0 & MASK]
        k0 = (k0 + W0) & MASK
        k1 = (k1 + W1) & MASK
    return c


KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((MASK, MASK, MASK, MASK), (MASK, MASK), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def _raw(records):
    from advanced_optimizers_b200 import _lib as L
    inp = torch.tensor(np.asarray(records, np.uint32).view(np.int32), device="cuda")
    out = torch.empty(len(records) * 4, dtype=torch.int32, device="cuda")
    L.check(L.lib().advopt_philox4x32_10(inp.data_ptr(), out.data_ptr(), len(records),
                                         torch.cuda.current_stream().cuda_stream), "philox")
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint32).reshape(-1, 4)


def test_philox_known_answers():
    got = _raw([list(c) + list(k) for c, k, _ in KAT])
    for (c, k, want), g in zip(KAT, got):
        assert tuple(int(x) for x in g) == want
        assert tuple(philox_py(c, k)) == want


def test_philox_matches_restatement():
    rng = np.random.default_rng(3)
    recs = rng.integers(0, 2 ** 32, size=(4096, 6), dtype=np.uint64).astype(np.uint32)
    got = _raw(recs)
    for r, g in zip(recs[:256], got[:256]):
        assert tuple(int(x) for x in g) == tuple(philox_py([int(v) for v in r[:4]], [int(r[4]), int(r[5])]))


def test_noise_fill_mapping_and_uniformity():
    from advanced_optimizers_b200 import _lib as L
    n = 1 << 20
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    seed, tid, step, stream = 42, 7, 3, 2
    L.check(L.lib().advopt_noise_fill(out.data_ptr(), n, seed, tid, step, stream,
                                      torch.cuda.current_stream().cuda_stream), "noise")
    torch.cuda.synchronize()
    r = out.cpu().numpy().view(np.uint16).astype(np.int64)
    for k0 in (0, 8, 8 * 12345):
        w = philox_py([k0 >> 3, (stream << 24), tid, step], [seed & MASK, seed >> 32])
        want = [w[e >> 1] >> (16 * (e & 1)) & 0xFFFF for e in range(8)]
        assert list(r[k0:k0 + 8]) == want
    hist = np.bincount(r >> 8, minlength=256)
    exp = n / 256
    chi2 = float(((hist - exp) ** 2 / exp).sum())
    assert chi2 < 255 + 6 * np.sqrt(2 * 255), chi2     # 255 dof, about 6 sigma
    assert abs(r.mean() - 32767.5) < 6 * 18918.6 / np.sqrt(n)


def test_bf16_stochastic_rounding_is_unbiased():
    import advanced_optimizers_b200 as A
    from oracle import oracle as O
    n = 1 << 20
    p = torch.nn.Parameter(torch.ones(n, dtype=torch.bfloat16, device="cuda"))
    opt = A.AdamW_adv([p], lr=1e-3, state_precision="fp32")
    p.grad = torch.full((n,), 1e-3, dtype=torch.bfloat16, device="cuda")
    opt.step()
    torch.cuda.synchronize()
    # the fp32 result before rounding: the same step on an fp32 parameter
    g1 = O.round_bf16(np.full(1, 1e-3, np.float32))
    hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, precision="fp32")
    st = O.adamw_init_state((1,), "f32", "fp32", False, 0.9)
    x = float(O.adam_family_step(np.ones(1, np.float32), "f32", g1, st, hp, {})[0])
    # bf16 neighbours of x (x > 0): truncation and the next bf16 value up
    bits_lo = int(np.float32(x).view(np.uint32)) & 0xFFFF0000
    lo = float(np.uint32(bits_lo).view(np.float32))
    hi = float(np.uint32(bits_lo + 0x10000).view(np.float32))
    vals = p.detach().float().cpu().numpy()
    assert set(np.unique(vals).tolist()) <= {lo, hi}
    want = (x - lo) / (hi - lo)
    got = float(np.mean(vals == hi))
    sigma = np.sqrt(want * (1 - want) / n)
    assert 0.05 < want < 0.95
    assert abs(got - want) <= 5 * sigma, (got, want, sigma)


def test_int8_quantisation_is_unbiased():
    import advanced_optimizers_b200 as A
    n = 1 << 20
    p = torch.nn.Parameter(torch.zeros(n, dtype=torch.bfloat16, device="cuda"))
    opt = A.AdamW_adv([p], lr=1e-3, state_precision="int8_sr")
    g = (torch.linspace(0.3, 1.0, n, device="cuda") * 1e-3).to(torch.bfloat16)
    p.grad = g
    opt.step()
    torch.cuda.synchronize()
    st = opt.state[p]
    codes = st["exp_avg"].float()
    scale = st["exp_avg_scale"].repeat_interleave(2048)[:n]
    m = 0.1 * g.float()     # lerp(0, g, 0.1), exact to within one float rounding
    err = (codes * scale - m).double()
    # per-element rounding error is uniform-like with variance <= scale^2 / 4
    sigma = float(torch.sqrt((scale.double() ** 2 / 4).sum())) / n
    assert abs(float(err.mean())) <= 5 * sigma + 1e-12, (float(err.mean()), sigma)
    assert float(err.abs().max()) <= float(scale.max()) * 1.0001
