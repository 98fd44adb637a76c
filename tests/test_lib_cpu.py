"""CPU-side checks of the native boundary: the library loads without a GPU,
exports every entry point include/advopt.h declares, and the Python struct
layouts match the C ones."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_symbols_exported():
    from advanced_optimizers_b200 import _lib
    L = _lib.lib()   # also checks ABI version and struct sizes
    hdr = open(os.path.join(ROOT, "include", "advopt.h")).read()
    declared = set(re.findall(r"\b(advopt_[a-z0-9_]+)\s*\(", hdr))
    assert declared, "no entry points parsed from advopt.h"
    for name in sorted(declared):
        assert hasattr(L, name), f"{name} declared in advopt.h but not exported"
    assert set(_lib.exported_symbols()) <= declared


def test_struct_sizes():
    from advanced_optimizers_b200 import _lib
    L = _lib.lib()
    assert L.advopt_sizeof(0) == _lib.ADAM_TENSOR_DT.itemsize == 232
    assert L.advopt_sizeof(1) == _lib.PIECE_DT.itemsize == 24
    assert L.advopt_sizeof(2) == ctypes.sizeof(_lib.AdamLaunch)
    assert L.advopt_sizeof(3) == _lib.LION_TENSOR_DT.itemsize


def test_invalid_launch_is_an_error_not_a_crash():
    from advanced_optimizers_b200 import _lib
    L = _lib.lib()
    s = _lib.AdamLaunch()
    rc = L.advopt_adam_step(ctypes.byref(s), None)
    assert rc == -1
    assert b"null table" in L.advopt_last_error()


@pytest.mark.parametrize("shapes", [
    [(96, 48), (48,), (50, 7), (2304,)],
    [(8192, 7168), (4096,), (128256, 4096)],
    [(3,), (2049,), (4097, 3), (1,)],
])
@pytest.mark.parametrize("grid", [1, 7, 148, 444])
def test_planner_covers_every_element_once(shapes, grid):
    from advanced_optimizers_b200._plan import effective_shape, plan, unit_of, CHUNK
    numels = [int(np.prod(s)) for s in shapes]
    d2s = [effective_shape(n)[1] if len(s) == 2 else 0 for s, n in zip(shapes, numels)]
    pieces, offsets, n_slots = plan(numels, d2s, grid)
    assert len(offsets) == grid + 1 and offsets[0] == 0 and offsets[-1] == len(pieces)
    assert np.all(np.diff(offsets) >= 0)
    covered = [0] * len(numels)
    for t in range(len(numels)):
        ps = pieces[pieces["tensor"] == t]
        ps = ps[np.argsort(ps["begin"])]
        pos = 0
        for pc in ps:
            assert pc["begin"] == pos
            assert pc["begin"] % CHUNK == 0
            if d2s[t]:
                assert pc["begin"] % d2s[t] == 0 and (pc["end"] % d2s[t] == 0)
            pos = pc["end"]
        covered[t] = pos
        assert sorted(ps["slot"].tolist()) == list(range(n_slots[t]))
    assert covered == numels


def test_state_dict_round_trip_keeps_exact_states_cpu():
    """load_state_dict keeps every saved state's dtype and value (torch alone
    would round float32 scales and factors of bf16 params to bf16), and the
    auxiliary Adam states of Muon keep their own precision."""
    import torch
    import advanced_optimizers_b200 as A
    g = torch.Generator().manual_seed(0)
    p = [torch.nn.Parameter(torch.randn(256, 64, generator=g).bfloat16()), torch.nn.Parameter(torch.randn(64).bfloat16())]
    o = A.AdamW_adv(p, state_precision="int8_sr", factored_2nd=True)
    for st in o.state.values():
        for k, v in st.items():
            if torch.is_tensor(v) and v.is_floating_point():
                v.copy_(torch.rand(v.shape, generator=g) + 0.1234567)
    sd = o.state_dict()
    q = [torch.nn.Parameter(t.detach().clone()) for t in p]
    o2 = A.AdamW_adv(q, state_precision="int8_sr", factored_2nd=True)
    o2.load_state_dict(sd)
    for a, b in zip(p, q):
        for k, v in o.state[a].items():
            if torch.is_tensor(v):
                w = o2.state[b][k]
                assert w.dtype == v.dtype, k
                assert torch.equal(w, v), k
    m = [torch.nn.Parameter(torch.randn(64, 48, generator=g).bfloat16()), torch.nn.Parameter(torch.randn(48).bfloat16())]
    mo = A.Muon_adv([dict(params=[m[0]], optim_type="muon"), dict(params=[m[1]], optim_type="adam")],
                    state_precision="int8_sr")
    sd = mo.state_dict()
    m2 = [torch.nn.Parameter(t.detach().clone()) for t in m]
    mo2 = A.Muon_adv([dict(params=[m2[0]], optim_type="muon"), dict(params=[m2[1]], optim_type="adam")],
                     state_precision="int8_sr")
    mo2.load_state_dict(sd)
    assert mo2.state[m2[1]]["exp_avg"].dtype == torch.bfloat16       # adam_state_precision 'auto'
    assert mo2.state[m2[0]]["momentum_buffer"].dtype == torch.int8
