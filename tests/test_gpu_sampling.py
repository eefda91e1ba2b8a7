"""On-device posterior sampling (act_mf_batch.stddev): the drawn clean / noise windows are the
Philox4x32-10 + Box-Muller draws of the restatement in test_philox.py for (seed, window, element),
a window draws the same values wherever it sits in a batch, and the step on them matches the CPU
oracle."""
import numpy as np
import pytest

from cases import MfCase
from test_philox import box_muller, philox4x32_10

pytestmark = pytest.mark.gpu


def expected(mean, std, seed, window0):
    n, lat, T = mean.shape
    per = lat * T
    clean = np.empty((n, per))
    noise = np.empty((n, per))
    for b in range(n):
        w = window0 + b
        words = [x for p in range((per + 1) // 2)
                 for x in philox4x32_10((p, w & 0xFFFFFFFF, w >> 32, 0x4D46), (seed & 0xFFFFFFFF, seed >> 32))]
        z = box_muller(words)[:2 * per].reshape(-1, 2)
        clean[b] = mean[b].reshape(-1).astype(np.float64) + std[b].reshape(-1) * z[:, 0]
        noise[b] = z[:, 1]
    return clean.reshape(mean.shape), noise.reshape(mean.shape)


def test_device_draws_follow_the_counter_based_generator():
    case = MfCase(seed=60, batch=3)
    mean, _, hidden, t, unc, valid = case.inputs()
    rng = np.random.default_rng(1)
    std = (0.05 + 0.3 * rng.random(mean.shape)).astype(np.float32)
    seed, w0 = 0x1234_5678_9ABC, (1 << 33) + 7
    loss = case.ctx.mf_step(mean, None, hidden, t, unc, valid, stddev=std, sample_seed=seed, window0=w0)
    g = case.ctx.get_grads()
    lat, T = mean.shape[1], mean.shape[2]
    dc, dz = case.ctx.mf_staged(3, lat, T)
    ec, ez = expected(mean, std, seed, w0)
    np.testing.assert_allclose(dc, ec, rtol=1e-5, atol=2e-6)  # libm ulps between device and host
    np.testing.assert_allclose(dz, ez, rtol=1e-5, atol=2e-6)
    assert abs(dz.mean()) < 0.05 and abs(dz.var() - 1) < 0.05
    # the step ran on exactly those draws
    ref_loss, ref_g = case.oracle(case.params, (dc, dz, hidden, t, unc, valid))
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-3)
    cos = float(np.dot(g, ref_g) / (np.linalg.norm(g) * np.linalg.norm(ref_g)))
    assert cos >= 0.9999, cos
    # a window draws the same values in another batch position; another seed draws others
    case.ctx.zero_grads()
    case.ctx.mf_step(mean[1:], None, hidden[1:], t[1:], unc[1:], valid[1:], stddev=std[1:], sample_seed=seed,
                     window0=w0 + 1)
    dc2, dz2 = case.ctx.mf_staged(2, lat, T)
    np.testing.assert_array_equal(dc2, dc[1:])
    np.testing.assert_array_equal(dz2, dz[1:])
    case.ctx.zero_grads()
    case.ctx.mf_step(mean, None, hidden, t, unc, valid, stddev=std, sample_seed=seed + 1, window0=w0)
    dc3, _ = case.ctx.mf_staged(3, lat, T)
    assert not np.array_equal(dc3, dc)


def test_sampling_with_a_bridge_is_rejected():
    import actrain as A
    case = MfCase(seed=61, batch=2)
    mean, _, hidden, t, unc, valid = case.inputs(n=2)
    with pytest.raises(A.ActError):
        case.ctx.mf_step(mean, None, hidden, t, unc, valid, pivot=mean, edit_start=np.zeros(2, np.float32),
                         stddev=np.ones_like(mean))
