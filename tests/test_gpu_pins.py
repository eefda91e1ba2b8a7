"""Bit-exact pins of the library's own integer / format work on the device, and the failure path
of a bounded device wait -- all through the C ABI.

* Q8_0: the device dequantisation that act_bind_weight runs (fp32 d*q, then the f16 GEMM
  operand) against gguf-py's Q8_0.dequantize_blocks goldens (tests/golden/q8_0.npz), bit for bit.
  Format: tools/ac-quantize.cpp:161,204 (34-byte blocks, fp16 d, int8 q[32]).
* Delay pattern: the delayed ids and scored targets that act_mg_stage puts on the device against
  the reference's tests/pattern_test.cpp:93-146 arrays (tests/golden/pattern_goldens.json),
  exactly; build_pattern_sequence of src/mg/pattern.h:64-76 and the target selection of
  src/mg/train.h:195-205.
* Bounded waits: a kernel waiting on a flag that nothing sets gives up after its limit, the call
  returns ACT_ERR_CUDA, and the context keeps working.
"""
import json
import os

import numpy as np
import pytest

import actrain as A
from cases import MfCase, MgCase, grad_metrics

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _f16_rne(x):
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)


def test_q8_0_device_dequantisation_is_bit_exact():
    g = np.load(os.path.join(GOLDEN, "q8_0.npz"))
    f32, h = A.q8_0_dequant(g["q"])
    want = g["deq"].astype(np.float32).ravel()
    np.testing.assert_array_equal(f32.view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(h, _f16_rne(want))


def _pattern_cases():
    return json.load(open(os.path.join(GOLDEN, "pattern_goldens.json")))["cases"]


@pytest.mark.parametrize("tag", ["MG", "ONE", "THREE"])
@pytest.mark.parametrize("prefix", [0, 1])
def test_staged_delay_pattern_matches_reference_goldens(tag, prefix):
    c = _pattern_cases()[tag]
    nq, T, S, special = c["n_q"], c["T"], c["S"], c["special"]
    if prefix >= T:
        pytest.skip("prefix must leave a scored frame")
    case = MgCase(dim=128, layers=1, heads=2, ff=256, n_q=nq, card=special, frames=T, C=8, prefix=prefix,
                  batch=1, dora=False, seed=30)
    codes = np.array(c["codes"], np.int32).reshape(1, nq, T)
    ctx = np.random.default_rng(0).standard_normal((1, 8, 128)).astype(np.float32)
    case.ctx.mg_stage(codes, ctx)
    ids, tgt = case.ctx.mg_staged(1, nq, S - 1, T - prefix)
    seq = np.array(c["sequence"], np.int32).reshape(nq, S)
    mask = np.array(c["mask"], np.int32).reshape(nq, S)
    # inputs are the pattern sequence without its last step
    np.testing.assert_array_equal(ids[0], seq[:, :S - 1])
    for q in range(nq):
        # scored rows: s whose next step holds a real code of timestep >= prefix
        rows = [s for s in range(S - 1) if mask[q, s + 1] and s + 1 - 1 - q >= prefix]
        assert len(rows) == T - prefix
        np.testing.assert_array_equal(tgt[0, q], seq[q, [s + 1 for s in rows]])
        np.testing.assert_array_equal(tgt[0, q], codes[0, q, prefix:])


def test_timed_out_wait_returns_an_error_and_the_context_keeps_working():
    case = MfCase(seed=40)
    with pytest.raises(A.ActError) as err:
        case.ctx.wait_probe(2_000_000)  # 2 ms on a flag nothing sets
    assert err.value.code == A.ACT_ERR_CUDA
    assert "code 99" in str(err.value)
    inp = case.inputs()
    loss = case.ctx.mf_step(*inp)
    ref_loss, ref_g = case.oracle(case.params, inp)
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-3)
    cos, rel, _, _ = grad_metrics(case.ctx.get_grads(), ref_g, case.layout)
    assert cos >= 0.9999 and rel <= 1e-2
