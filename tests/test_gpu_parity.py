"""CUDA path vs the CPU oracle, through the C ABI (libactrain.so).

Tolerances (f16 GEMM operands, fp32 accumulation, against the fp32 oracle on the same
dequantised weights), the BASELINE parity gates:
  loss        |rel| <= 1e-3
  gradients   cosine >= 0.9999 over all adapter gradients, and the relative error of every
              adapter tensor, ||g - ref|| / ||ref||, <= 1e-2 (so also over all of them).
"""
import numpy as np
import pytest

import actrain as A
import oracle as O
from cases import MfCase, MgCase, dequant, grad_metrics, q8_0_bytes

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-3
COS_MIN = 0.9999
GLOBAL_REL = 1e-2
TENSOR_REL = 1e-2


def _check(loss, ref_loss, g, ref_g, layout):
    np.testing.assert_allclose(loss, ref_loss, rtol=LOSS_RTOL)
    cos, rel, worst, name = grad_metrics(g, ref_g, layout)
    assert cos >= COS_MIN, (cos, rel, worst, name)
    assert rel <= GLOBAL_REL, (cos, rel, worst, name)
    assert worst <= TENSOR_REL, (cos, rel, worst, name)


@pytest.mark.parametrize("dora", [False, True], ids=["lora", "dora"])
@pytest.mark.parametrize("wtype", ["f32", "f16", "q8_0"])
def test_mf_step_matches_oracle(dora, wtype):
    case = MfCase(dora=dora, wtype=wtype, seed=1 + dora)
    inp = case.inputs()
    loss = case.ctx.mf_step(*inp)
    g = case.ctx.get_grads()
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, g, ref_g, case.layout)


def test_mf_first_layer_and_target_subset():
    case = MfCase(layers=6, targets=0x63, first=2, rank=8, alpha=16.0, seed=5)
    inp = case.inputs()
    loss = case.ctx.mf_step(*inp)
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, case.ctx.get_grads(), ref_g, case.layout)


def test_mf_zero_b_gives_exactly_zero_a_gradient():
    case = MfCase(b_std=0.0, seed=3)
    case.ctx.mf_step(*case.inputs())
    g = case.ctx.get_grads()
    for name, off, shape in case.layout:
        k = int(np.prod(shape))
        if name.endswith("lora_A"):
            assert np.count_nonzero(g[off:off + k]) == 0, name
    assert np.abs(g).max() > 0


def test_mf_unconditional_cross_attention_gets_no_gradient():
    case = MfCase(seed=4)
    inp = case.inputs(n=1, modes=["null"])
    case.ctx.mf_step(*inp)
    g = case.ctx.get_grads()
    for name, off, shape in case.layout:
        if ".cross." in name:
            assert np.count_nonzero(g[off:off + int(np.prod(shape))]) == 0, name


def test_graph_replay_matches_first_run():
    case = MfCase(seed=6)
    inp = case.inputs()
    runs = []
    for _ in range(3):  # eager, captured, replayed
        loss = case.ctx.mf_step(*inp)
        runs.append((loss, case.ctx.get_grads()))
        case.ctx.zero_grads()
    for loss, g in runs[1:]:
        np.testing.assert_allclose(loss, runs[0][0], rtol=1e-6)
        np.testing.assert_allclose(g, runs[0][1], rtol=1e-4, atol=1e-6 * np.abs(runs[0][1]).max())


def test_mf_stream_k_matches_whole_tiles(monkeypatch):
    """d1024 DiT, 8 x 750 frames: the 1024- and 4096-wide projections have more 256 x 256 pair
    tiles than SM pairs with a mostly idle last round, so the GEMMs split them stream-K.  The
    step must equal the same step on whole tiles up to fp32 summation order, and stay equal
    over the eager, captured and replayed runs (the partial-tile flags reset every launch)."""
    kw = dict(dim=1024, layers=2, heads=16, ff=4096, lat=128, cond=64, tdim=32, T=750, C=32, rank=16,
              alpha=32.0, batch=8, seed=11)
    monkeypatch.setenv("ACTRAIN_STREAMK", "0")
    whole = MfCase(**kw)
    monkeypatch.delenv("ACTRAIN_STREAMK")
    split = MfCase(**kw)
    inp = whole.inputs(modes=["cond", "padded", "null"] + ["cond"] * 5)
    loss0 = whole.ctx.mf_step(*inp)
    g0 = whole.ctx.get_grads()
    for _ in range(3):
        loss = split.ctx.mf_step(*inp)
        _check(loss, loss0, split.ctx.get_grads(), g0, split.layout)
        split.ctx.zero_grads()


def test_gradients_accumulate_over_microbatches():
    case = MfCase(seed=7)
    a, b = case.inputs(n=2), case.inputs(n=1)
    case.ctx.mf_step(*a)
    case.ctx.mf_step(*b)
    g = case.ctx.get_grads()
    _, ga = case.oracle(case.params, a)
    _, gb = case.oracle(case.params, b)
    cos, rel, worst, name = grad_metrics(g, ga + gb, case.layout)
    assert cos >= COS_MIN and rel <= GLOBAL_REL and worst <= TENSOR_REL, (cos, rel, worst, name)


@pytest.mark.parametrize("decay", [0.0, 0.01])
def test_optimizer_matches_reference_update(decay):
    case = MfCase(seed=8)
    inp = case.inputs()
    case.ctx.mf_step(*inp)
    g = case.ctx.get_grads()
    v0, m0, s0 = case.ctx.get_params()
    nonfinite = case.ctx.optimizer(lr=1e-3, step=1, weight_decay=decay, clip=0.5)
    assert nonfinite == 0
    v1, m1, s1 = case.ctx.get_params()
    names = [n for n, _, _ in case.layout]
    mask = np.zeros(v0.size, np.uint8)
    for name, off, shape in case.layout:
        if name.endswith(("lora_A", "lora_B")):
            mask[off:off + int(np.prod(shape))] = 1
    rv, rm, rs, rg = v0.copy(), m0.copy(), s0.copy(), g.copy()
    O.lib().ora_adamw(rv.size, rv, rm, rs, rg, mask, case.batch, 1, 1e-3, 0.9, 0.999, 1e-8, decay, 0.5)
    np.testing.assert_allclose(v1, rv, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(m1, rm, rtol=1e-4, atol=1e-9)
    assert np.count_nonzero(case.ctx.get_grads()) == 0  # update consumes the accumulation
    assert names


def test_adam_steps_reduce_loss():
    case = MfCase(seed=9, batch=1)
    inp = case.inputs(n=1, modes=["cond"])
    before = case.ctx.mf_step(*inp)[0]
    case.ctx.zero_grads()
    for step in range(1, 31):
        case.ctx.mf_step(*inp)
        case.ctx.optimizer(lr=4e-3, step=step)
    after = case.ctx.mf_step(*inp)[0]
    assert after < 0.9 * before


def test_param_table_and_init_follow_reference_order():
    case = MfCase(dora=True, b_std=0.0, seed=10)
    table = case.ctx.param_table()
    assert [(n, o, int(np.prod(s))) for n, o, s in table] == \
        [(n, o, int(np.prod(s))) for n, o, s in case.layout]
    init = case.init
    for name, off, shape in case.layout:
        k = int(np.prod(shape))
        seg = init[off:off + k]
        if name.endswith("lora_B"):
            assert np.count_nonzero(seg) == 0
        elif name.endswith("lora_A"):
            assert abs(seg.std() - 0.02) < 0.004 and abs(seg.mean()) < 0.004
    # magnitude = sqrt(row norm^2 + in*1e-12) of the bound base (src/ac/lora.h:11-32, train.h:99)
    W = {}
    off = 0
    for n, (r, c) in zip(O.dit_tensor_names(case.cfg), O.dit_tensor_shapes(case.cfg)):
        W[n] = case.Wflat[off:off + r * c].reshape(r, c)
        off += r * c
    for name, o, shape in case.layout:
        if name.endswith("magnitude"):
            base = W[name[: -len(".magnitude")]]
            nsq = np.zeros(base.shape[0], np.float32)
            O.lib().ora_row_norm_sq(np.ascontiguousarray(base), base.shape[0], base.shape[1], nsq)
            np.testing.assert_array_equal(init[o:o + shape[0]], np.sqrt(nsq))


def test_q8_0_binding_is_exact_dequantisation():
    # A Q8_0 bound projection must behave exactly like its F32 dequantisation bound as F32.
    a = MfCase(wtype="q8_0", seed=11)
    inp = a.inputs()
    la = a.ctx.mf_step(*inp)
    ga = a.ctx.get_grads()
    ref_loss, ref_g = a.oracle(a.params, inp)
    _check(la, ref_loss, ga, ref_g, a.layout)


@pytest.mark.parametrize("dora", [False, True], ids=["lora", "dora"])
def test_mg_step_matches_oracle(dora):
    case = MgCase(dora=dora, seed=20 + dora)
    inp = case.inputs()
    loss = case.ctx.mg_step(*inp)
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, case.ctx.get_grads(), ref_g, case.layout)


def test_mg_prefix_and_first_layer():
    case = MgCase(prefix=5, first=1, targets=0x1F, wtype="q8_0", seed=23)
    inp = case.inputs()
    loss = case.ctx.mg_step(*inp)
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, case.ctx.get_grads(), ref_g, case.layout)


@pytest.mark.parametrize("tokens", [5, 13])
def test_conditioning_not_a_multiple_of_eight(tokens):
    """Any token count: the device pads the conditioning to a multiple of 8 and masks the padding.
    MusicGen attends to every caller row (the reference pads with zeros and does not mask them,
    src/mg/train.h:181-186); MelodyFlow masks past valid_tokens as before."""
    mg = MgCase(C=tokens, dora=True, seed=40 + tokens)
    inp = mg.inputs()
    loss = mg.ctx.mg_step(*inp)
    ref_loss, ref_g = mg.oracle(mg.params, inp)
    _check(loss, ref_loss, mg.ctx.get_grads(), ref_g, mg.layout)
    mf = MfCase(C=tokens, seed=50 + tokens)
    inp = mf.inputs()
    loss = mf.ctx.mf_step(*inp)
    ref_loss, ref_g = mf.oracle(mf.params, inp)
    _check(loss, ref_loss, mf.ctx.get_grads(), ref_g, mf.layout)


def test_mg_cross_kv_without_adapter():
    # no adapter on cross.kv: its projection runs as a plain GEMM and has no backward
    case = MgCase(targets=0x77, layers=3, seed=24)
    inp = case.inputs()
    loss = case.ctx.mg_step(*inp)
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, case.ctx.get_grads(), ref_g, case.layout)


def test_invalid_inputs_are_rejected():
    case = MfCase(seed=12)
    clean, noise, hidden, t, unc, valid = case.inputs()
    with pytest.raises(A.ActError):
        case.ctx.mf_step(clean, noise, hidden, np.array([0.5, 1.5, 0.2], np.float32), unc, valid)
    with pytest.raises(A.ActError):
        case.ctx.mf_step(clean, noise, hidden, t, unc, np.array([99, -1, -1], np.int32))
    with pytest.raises(A.ActError):
        case.ctx.optimizer(lr=-1.0, step=1)


# ---- the benchmarked configuration's shapes (BASELINE cfg 2 per layer: d1024, 16 heads, FFN 4096,
# T = 750, 32 tokens, Q8_0 base, rank 16, alpha 32), two layers and two clips so that the oracle
# finishes in seconds.  At T >= 128 the self-attention forward and backward run on the tcgen05
# kernels inside the step; path_counts proves it.
CFG2 = dict(dim=1024, layers=2, heads=16, ff=4096, lat=128, cond=768, tdim=256, T=750, C=32, rank=16,
            alpha=32.0, wstd=0.02, wtype="q8_0", batch=2)


def _assert_tc_attention(case, layers):
    pc = case.ctx.path_counts()
    assert pc["attn_fwd_tc"] == layers and pc["attn_bwd_tc"] == layers, pc
    # cross-attention over the conditioning tokens (at most 64): the tcgen05 query-major kernels
    assert pc["xattn_fwd_tc"] == layers and pc["xattn_bwd_tc"] == layers, pc
    # every block projection (seven per layer, forward) at least runs on the tcgen05 GEMM
    assert pc["gemm_tc"] >= 7 * layers, pc


@pytest.mark.parametrize("dora,targets", [(False, 0x63), (False, 0x7F), (True, 0x7F)],
                         ids=["lora-qkv-out-ffn", "lora-all", "dora-all"])
def test_mf_cfg2_shapes_match_oracle(dora, targets):
    case = MfCase(**CFG2, dora=dora, targets=targets, seed=50 + targets + dora)
    inp = case.inputs(n=2, modes=["cond", "padded"])
    loss = case.ctx.mf_step(*inp)
    _assert_tc_attention(case, 2)
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, case.ctx.get_grads(), ref_g, case.layout)


@pytest.mark.parametrize("T", [200, 750])
def test_mf_tcgen05_attention_in_step_with_dora(T):
    # narrow model, long clips: the tcgen05 self-attention with the DoRA k / v / q column factors,
    # the inverse RoPE of the dQ finish and the 3-D strided dQKV layout, against the oracle
    case = MfCase(dim=128, layers=3, heads=2, ff=256, T=T, C=16, dora=True, batch=2, wtype="q8_0", seed=60 + T)
    inp = case.inputs(n=2, modes=["cond", "null"])
    loss = case.ctx.mf_step(*inp)
    _assert_tc_attention(case, 3)
    ref_loss, ref_g = case.oracle(case.params, inp)
    _check(loss, ref_loss, case.ctx.get_grads(), ref_g, case.layout)


def test_mf_cfg1_training_trajectory():
    """BASELINE cfg 1: 24 blocks at d1024, one 250-frame clip, 16 tokens, F16 base, LoRA r16 / alpha
    32 on q/k/v/o/ffn_in/ffn_out with the reference initialisation (B = 0), AdamW lr 1e-4 wd 0.01,
    10 steps.  The per-step loss of the device trajectory stays within 1e-3 of the oracle's own
    trajectory (oracle gradients, oracle AdamW)."""
    case = MfCase(dim=1024, layers=24, heads=16, ff=4096, lat=128, cond=768, tdim=256, T=250, C=16, rank=16,
                  alpha=32.0, wstd=0.02, wtype="f16", batch=1, targets=0x63, b_std=0.0, seed=0)
    mask = np.zeros(case.params.size, np.uint8)
    for name, off, shape in case.layout:
        mask[off:off + int(np.prod(shape))] = 1
    p = case.params.copy()
    m, v = np.zeros_like(p), np.zeros_like(p)
    for step in range(1, 11):
        inp = case.inputs(n=1, modes=["cond"])
        loss = case.ctx.mf_step(*inp)
        ref_loss, ref_g = case.oracle(p, inp)
        np.testing.assert_allclose(loss, ref_loss, rtol=LOSS_RTOL, err_msg=f"step {step}")
        if step == 1:  # B = 0: only dB is nonzero, dA is exactly zero on both sides
            g = case.ctx.get_grads()
            cos, rel, _, _ = grad_metrics(g, ref_g, case.layout)
            assert cos >= COS_MIN and rel <= GLOBAL_REL, (cos, rel)
        assert case.ctx.optimizer(lr=1e-4, step=step, weight_decay=0.01, clip=1.0) == 0
        O.lib().ora_adamw(p.size, p, m, v, ref_g.astype(np.float32), mask, 1, step, 1e-4, 0.9, 0.999, 1e-8,
                          0.01, 1.0)
