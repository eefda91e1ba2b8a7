"""With act_set_deterministic the step is bit-for-bit reproducible: the same microbatch gives the
same losses and gradients on every run.  The reference's CPU graph is deterministic and mf-train / mg-train rely on it
(exact resume from a .state file, checkpoints that leave the trained weights unchanged:
src/ac/train_controls.h:122-196, tools/mf-train.cpp:300-346), so no reduction on the device may
depend on the order in which CTAs finish.  The shapes make every split reduction run with several
partials: the rank-block products (split-K over rows), the DoRA column sums, the cross-attention
query split and the MusicGen cross-entropy rows."""
import numpy as np
import pytest

from cases import MfCase, MgCase

pytestmark = pytest.mark.gpu


def _twice(step, get):
    out = []
    for _ in range(2):
        step_out = step()
        out.append((np.array(step_out, copy=True), get()))
    return out


@pytest.mark.parametrize("dora,T", [(False, 200), (True, 200), (False, 640)], ids=["lora", "dora", "lora-T640"])
def test_mf_step_is_reproducible(dora, T):
    # T = 640: five 128-key blocks add into every query block's dQ (the ordered adds)
    case = MfCase(dim=256, heads=4, ff=512, T=T, C=24, rank=8, alpha=16.0, dora=dora, batch=3, seed=31)
    case.ctx.set_deterministic(True)
    inp = case.inputs()

    def step():
        case.ctx.zero_grads()
        return case.ctx.mf_step(*inp)

    (l1, g1), (l2, g2) = _twice(step, case.ctx.get_grads)
    np.testing.assert_array_equal(l1, l2)
    np.testing.assert_array_equal(g1, g2)
    assert np.count_nonzero(g1) > g1.size // 2


def test_mg_step_is_reproducible():
    case = MgCase(dim=256, heads=4, ff=512, frames=600, card=128, dora=True, batch=2, seed=32)
    case.ctx.set_deterministic(True)
    inp = case.inputs()

    def step():
        case.ctx.zero_grads()
        return case.ctx.mg_step(*inp)

    (l1, g1), (l2, g2) = _twice(step, case.ctx.get_grads)
    np.testing.assert_array_equal(l1, l2)
    np.testing.assert_array_equal(g1, g2)
