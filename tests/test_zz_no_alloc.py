"""Attention backward that allocates nothing (act_attention_bwd_noalloc) against the regular
entry point (act_attention) on the same inputs.

The no-allocation entry point is for callers that may not call cudaMalloc: real-time hosts such
as an audio plug-in's processing thread, code recording a CUDA graph under global capture, and
embedders that own all device memory.  They pass device inputs and outputs; the backward's
scratch lives in a fixed array inside the library, shared by every call.  This file is named so
that pytest collects it last: if it fails, a stop-at-first-failure run has already run the rest.
"""
import numpy as np
import pytest
import torch

import actrain as A
from f16util import bits_to_f32, f16_bits

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2  # the attention tests' tolerance (relative L2, f16 outputs)


def _bits(x):
    return f16_bits(x)


def _f32(b):
    return bits_to_f32(np.ascontiguousarray(b).view(np.uint16)).astype(np.float64)


def _rope(T):
    ff = 10000.0 ** (2 * np.arange(32) / 64.0)
    th = (np.arange(T, dtype=np.float32)[:, None] / ff[None, :].astype(np.float32)).astype(np.float32)
    return np.ascontiguousarray(np.stack([np.cos(th), np.sin(th)], -1), np.float32)


def _dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to("cuda")


@pytest.mark.parametrize("case", [
    dict(clips=2, T=150, Tk=150, H=2, nvalid=None, causal=False, zero_key=True, rope=True),
    dict(clips=3, T=90, Tk=16, H=2, nvalid=[16, 5, 0], causal=False, zero_key=True, rope=False),
    dict(clips=1, T=200, Tk=200, H=3, nvalid=None, causal=True, zero_key=False, rope=False),
], ids=["self_rope", "cross_masked", "causal"])
def test_noalloc_backward_matches_act_attention_twice(case):
    c = case
    rng = np.random.default_rng(c["T"] + c["H"])
    D = c["H"] * 64
    q = _bits(rng.standard_normal((c["clips"] * c["T"], D)))
    k = _bits(rng.standard_normal((c["clips"] * c["Tk"], D)))
    v = _bits(rng.standard_normal((c["clips"] * c["Tk"], D)))
    do = _bits(rng.standard_normal((c["clips"] * c["T"], D)))
    tab = _rope(c["T"]) if c["rope"] else None
    ref = A.attention(q, k, v, do, c["clips"], c["T"], c["Tk"], c["H"], c["nvalid"], c["causal"], c["zero_key"], tab)

    dq_, dk_, dv_ = q, k, v  # output shapes
    ins = {n: _dev(a) for n, a in (("q", q), ("k", k), ("v", v), ("o", ref["o"]), ("lse", ref["lse"]), ("do", do))}
    nv = _dev(np.array(c["nvalid"], np.int32)) if c["nvalid"] is not None else None
    rp = _dev(tab) if tab is not None else None
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the shared scratch must be reset by every call
        outs = {n: torch.full(a.shape, 0x7F7F, dtype=torch.int16, device="cuda")
                for n, a in (("dq", dq_), ("dk", dk_), ("dv", dv_))}
        A.attention_bwd_noalloc(ins["q"].data_ptr(), ins["k"].data_ptr(), ins["v"].data_ptr(), ins["o"].data_ptr(),
                                ins["lse"].data_ptr(), ins["do"].data_ptr(), outs["dq"].data_ptr(),
                                outs["dk"].data_ptr(), outs["dv"].data_ptr(), c["clips"], c["T"], c["Tk"], c["H"],
                                nv.data_ptr() if nv is not None else 0, c["causal"], c["zero_key"],
                                rp.data_ptr() if rp is not None else 0, stream)
        torch.cuda.synchronize()
        for name in ("dq", "dk", "dv"):
            got = _f32(outs[name].cpu().numpy())
            want = _f32(ref[name])
            scale = np.linalg.norm(want)
            if scale == 0:
                assert np.count_nonzero(got) == 0, (call, name)
                continue
            rel = np.linalg.norm(got - want) / scale
            assert rel <= REL_TOL, (call, name, rel)


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    big = torch.zeros(16, dtype=torch.int16, device="cuda")  # never touched: rejected before launch
    p = big.data_ptr()
    with pytest.raises(A.ActError) as err:
        A.attention_bwd_noalloc(p, p, p, p, p, p, p, p, p, clips=64, T=3000, Tk=3000, H=24)
    assert err.value.code == A.ACT_ERR_INVALID
    assert "fixed maximum" in str(err.value)


def test_noalloc_rejects_misaligned_pointers():
    buf = torch.zeros(4096, dtype=torch.int16, device="cuda")  # never touched: rejected before launch
    p = buf.data_ptr()
    with pytest.raises(A.ActError) as err:
        A.attention_bwd_noalloc(p + 2, p, p, p, p, p, p, p, p, clips=1, T=64, Tk=64, H=1)
    assert err.value.code == A.ACT_ERR_INVALID
    assert "aligned" in str(err.value)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in one process")
def test_noalloc_on_a_second_device_in_the_same_process():
    # the scratch address and the kernels' shared-memory limits are set up per device
    c = dict(clips=2, T=150, Tk=150, H=2)
    rng = np.random.default_rng(7)
    D = c["H"] * 64
    q, k, v, do = (_bits(rng.standard_normal((c["clips"] * c["T"], D))) for _ in range(4))
    tab = _rope(c["T"])
    ref = A.attention(q, k, v, do, c["clips"], c["T"], c["Tk"], c["H"], None, False, True, tab, device=0)
    for dev in (0, 1):
        with torch.cuda.device(dev):
            ins = [_dev(a) for a in (q, k, v, ref["o"], ref["lse"], do)]
            rp = _dev(tab)
            outs = [torch.zeros(a.shape, dtype=torch.int16, device="cuda") for a in (q, k, v)]
            A.attention_bwd_noalloc(*[t.data_ptr() for t in ins], *[t.data_ptr() for t in outs], c["clips"], c["T"],
                                    c["Tk"], c["H"], 0, False, True, rp.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            for name, got in zip(("dq", "dk", "dv"), outs):
                want = _f32(ref[name])
                rel = np.linalg.norm(_f32(got.cpu().numpy()) - want) / np.linalg.norm(want)
                assert rel <= REL_TOL, (dev, name, rel)
