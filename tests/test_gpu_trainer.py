"""mf-train on the GPU: the reference CLI test's contract (tests/mf_train_cli_test.py of the reference:
evaluation and checkpoints leave training unchanged, exact resume, logit-normal time, DoRA rows,
the edit-bridge objective, rejected settings) on a DiT our kernels run, plus parity of the printed
losses with a replay of the same draws through the CPU oracle, and the library's bridge endpoint
against the host formula."""
import os
import re
import subprocess

import numpy as np
import pytest

import actrain as A
import oracle as O
import trainer_fixtures as TF

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "audiocraft.cpp_b200", "bin", "mf-train")
LOSS_REL = 1e-3  # north_star: loss within 1e-3 relative of the fp32 CPU path


@pytest.fixture(scope="module")
def world(tmp_path_factory):
    if not os.path.exists(EXE):
        pytest.skip("mf-train is not built")
    root = tmp_path_factory.mktemp("mftrain")
    dit = TF.TinyDit()
    dit.write(root / "base.gguf")
    TF.write_caches(root / "train", dit, 2, 52, seed=5, tokens=(5, 8), empty=(1,), captions=["warm synth pad"])
    TF.write_caches(root / "validation", dit, 2, 48, seed=6, tokens=(8, 3))
    TF.write_caches(root / "bridge_train", dit, 2, 48, seed=7, bridge_start=0.11)
    TF.write_caches(root / "bridge_validation", dit, 2, 48, seed=8, bridge_start=0.11)
    return root, dit


def run(root, *args):
    return subprocess.run([EXE, "--dit", str(root / "base.gguf"), *map(str, args)], capture_output=True, text=True,
                          timeout=600)


def common(root, cache="train", validation="validation"):
    return ["--cache", root / cache, "--validation", root / validation, "--frames", 48, "--rank", 4, "--first-layer",
            0, "--steps", 4, "--seed", 77]


def printed(stderr):
    before = float(re.search(r"probe before ([-0-9.]+)", stderr).group(1))
    steps = [float(x) for x in re.findall(r"\] step \d+/\d+ windows \d+ lr \S+ loss ([-0-9.]+)", stderr)]
    after = float(re.search(r"fixed probe after ([-0-9.]+)", stderr).group(1))
    return before, steps, after


def test_losses_follow_the_oracle_replay(world):
    """Same draws, same order: every loss mf-train prints is the oracle's within 1e-3 relative."""
    root, dit = world
    out = root / "parity.gguf"
    args = common(root) + ["--out", out, "--steps", 3, "--accumulation-steps", 2, "--random-crop", "--train-ffn",
                           "--cfg-dropout", 0.3, "--t-sampling", "logit-normal", "--t-mean", 0.2, "--warmup-steps", 2,
                           "--lr", 2e-3, "--weight-decay", 0.01, "--eval-samples", 0, "--eval-draws", 2, "--alpha", 8]
    r = run(root, *args)
    assert r.returncode == 0, r.stderr
    rep = TF.MfTrainReplay(dit, TF.read_caches(root / "train"), TF.read_caches(root / "validation"), 48, 4, 8.0, 0, 77,
                           0x7F, accumulation=2, dropout=0.3, random_crop=True, t_sampling="logit-normal", t_mean=0.2,
                           eval_samples=0, eval_draws=2, lr=2e-3, warmup=2, decay=0.01)
    want = rep.train(3)
    before, steps, after = printed(r.stderr)
    assert len(steps) == 3
    for got, ref in [(before, want["before"])] + list(zip(steps, want["steps"])) + [(after, want["after"])]:
        assert abs(got - ref) <= LOSS_REL * abs(ref) + 2e-7, (got, ref, r.stderr)
    params, meta = TF.read_adapter(out)
    assert meta["ac.lora.rank"] == 4 and meta["ac.lora.alpha"] == 8.0 and meta["ac.lora.type"] == "lora"
    assert meta["ac.lora.training_time_density"] == "logit-normal" and meta["ac.lora.base_name"] == "tiny test dit"
    got = np.concatenate([params[name] for name, _, _ in rep.layout])
    # AdamW moves every entry by about lr whatever its gradient's size, so an entry whose gradient
    # is near zero (and differs in sign between the fp32 CPU sum and the device's) steps the other
    # way: the parameters agree to a few 1e-3, the losses above to 1e-3
    assert np.linalg.norm(got - rep.params) <= 5e-3 * np.linalg.norm(rep.params)
    assert (root / "parity.prompts.json").exists() and (root / "parity.gguf.state").exists()


def test_evaluation_and_checkpoints_leave_training_unchanged(world):
    root, _ = world
    plain = run(root, *common(root), "--out", root / "plain.gguf")
    assert plain.returncode == 0, plain.stderr
    ck = run(root, *common(root), "--out", root / "checkpointed.gguf", "--eval-samples", 0, "--eval-draws", 3,
             "--checkpoint-every", 2)
    assert ck.returncode == 0, ck.stderr
    assert (root / "checkpointed.step-2.gguf").is_file() and "fixed probe step 2" in ck.stderr
    assert (root / "plain.gguf").read_bytes() == (root / "checkpointed.gguf").read_bytes()


def test_exact_resume_with_accumulation_warmup_decay_crops_and_ffn(world):
    root, _ = world
    controls = ["--accumulation-steps", 3, "--warmup-steps", 3, "--lr-schedule", "inverse", "--weight-decay", 0.01,
                "--beta2", 0.95, "--random-crop", "--train-ffn", "--frames", 40]
    full = run(root, *common(root), *controls, "--out", root / "controls.gguf", "--checkpoint-every", 2)
    assert full.returncode == 0, full.stderr
    resumed = run(root, *common(root), *controls, "--out", root / "resumed.gguf", "--checkpoint-every", 0,
                  "--resume", root / "controls.step-2.gguf.state")
    assert resumed.returncode == 0, resumed.stderr
    assert (root / "controls.gguf").read_bytes() == (root / "resumed.gguf").read_bytes()
    assert (root / "controls.gguf.state").read_bytes() == (root / "resumed.gguf.state").read_bytes()
    params, _ = TF.read_adapter(root / "controls.gguf")
    assert any(".ff.0." in n for n in params)
    changed = run(root, *common(root), *controls, "--out", root / "bad-resume.gguf", "--resume",
                  root / "controls.step-2.gguf.state", "--lr", 2e-4)
    assert changed.returncode != 0 and not (root / "bad-resume.gguf").exists()


def test_logit_normal_time_changes_training_but_not_the_probe(world):
    root, _ = world
    plain = root / "plain.gguf"
    if not plain.exists():
        assert run(root, *common(root), "--out", plain).returncode == 0
    base = run(root, *common(root), "--out", root / "plain-again.gguf")
    logit = run(root, *common(root), "--out", root / "logit.gguf", "--t-sampling", "logit-normal")
    checked = run(root, *common(root), "--out", root / "logit-checked.gguf", "--t-sampling", "logit-normal",
                  "--checkpoint-every", 2)
    assert base.returncode == 0 and logit.returncode == 0 and checked.returncode == 0, logit.stderr + checked.stderr
    assert (root / "logit.gguf").read_bytes() == (root / "logit-checked.gguf").read_bytes()
    assert (root / "logit.gguf").read_bytes() != plain.read_bytes()
    probe = lambda s: next(l for l in s.splitlines() if "probe before" in l)
    assert probe(logit.stderr) == probe(base.stderr)


def test_dora_rows_checkpoint_invariance(world):
    root, _ = world
    a = run(root, *common(root), "--out", root / "dora.gguf", "--adapter-type", "dora-rows", "--t-sampling",
            "logit-normal")
    b = run(root, *common(root), "--out", root / "dora-checked.gguf", "--adapter-type", "dora-rows", "--t-sampling",
            "logit-normal", "--checkpoint-every", 2)
    assert a.returncode == 0 and b.returncode == 0, a.stderr + b.stderr
    assert (root / "dora.gguf").read_bytes() == (root / "dora-checked.gguf").read_bytes()
    params, meta = TF.read_adapter(root / "dora.gguf")
    assert meta["ac.lora.type"] == "dora-rows" and any(n.endswith(".magnitude") for n in params)


def test_edit_bridge_objective(world):
    root, dit = world
    paired = common(root, "bridge_train", "bridge_validation") + ["--objective", "edit-bridge", "--t-min", 0.11,
                                                                   "--t-sampling", "logit-normal"]
    a = run(root, *paired, "--out", root / "bridge.gguf", "--steps", 3)
    b = run(root, *paired, "--out", root / "bridge-checked.gguf", "--steps", 3, "--checkpoint-every", 2)
    assert a.returncode == 0 and b.returncode == 0, a.stderr + b.stderr
    assert (root / "bridge.gguf").read_bytes() == (root / "bridge-checked.gguf").read_bytes()
    rep = TF.MfTrainReplay(dit, TF.read_caches(root / "bridge_train"), TF.read_caches(root / "bridge_validation"), 48,
                           4, 4.0, 0, 77, 0x1F, t_sampling="logit-normal", bridge=True)
    want = rep.train(3)
    before, steps, after = printed(a.stderr)
    for got, ref in [(before, want["before"])] + list(zip(steps, want["steps"])) + [(after, want["after"])]:
        assert abs(got - ref) <= LOSS_REL * abs(ref) + 2e-7, (got, ref)
    _, meta = TF.read_adapter(root / "bridge.gguf")
    assert meta["ac.lora.training_objective"] == "edit-bridge"
    wrong = run(root, *common(root), "--objective", "edit-bridge", "--out", root / "wrong.gguf")
    assert wrong.returncode != 0 and not (root / "wrong.gguf").exists()
    mismatch = run(root, *paired, "--t-min", 0.12, "--out", root / "mismatch.gguf")
    assert mismatch.returncode != 0 and not (root / "mismatch.gguf").exists()


def test_bridge_endpoint_on_the_device_matches_the_host_formula():
    """act_mf_batch.pivot / edit_start: the same losses and gradients as the plain step given the
    endpoint (pivot - start*clean)/(1 - start) computed on the host, bit for bit."""
    from cases import MfCase
    case = MfCase(seed=21, batch=3)
    clean, noise, hidden, t, unc, valid = case.inputs()
    rng = np.random.default_rng(4)
    pivot = rng.standard_normal(clean.shape).astype(np.float32)
    start = np.array([0.0, 0.25, 0.6], np.float32)
    t = np.maximum(t, start).astype(np.float32)
    s = start[:, None, None]
    endpoint = ((pivot - s * clean) / (np.float32(1) - s)).astype(np.float32)
    case.ctx.zero_grads()
    l1 = case.ctx.mf_step(clean, endpoint, hidden, t, unc, valid)
    g1 = case.ctx.get_grads()
    case.ctx.zero_grads()
    l2 = case.ctx.mf_step(clean, None, hidden, t, unc, valid, pivot=pivot, edit_start=start)
    g2 = case.ctx.get_grads()
    np.testing.assert_array_equal(l1, l2)
    np.testing.assert_array_equal(g1, g2)
    ref, _ = case.oracle(case.params, (clean, endpoint, hidden, t, unc, valid))
    np.testing.assert_allclose(l2, ref, rtol=LOSS_REL)
    case.ctx.zero_grads()
    bad = start.copy()
    bad[1] = 1.0
    with pytest.raises(A.ActError):
        case.ctx.mf_step(clean, None, hidden, t, unc, valid, pivot=pivot, edit_start=bad)
    with pytest.raises(A.ActError):  # t below the bridge start
        case.ctx.mf_step(clean, None, hidden, np.zeros(3, np.float32) + 0.1, unc, valid, pivot=pivot,
                         edit_start=np.full(3, 0.5, np.float32))


def test_device_sampling_is_resumable_and_checkpoint_invariant(world):
    """--device-sampling: the posterior and noise are drawn on the GPU per (seed, window), so a
    resumed run and a checkpointed run still write what the uninterrupted one writes."""
    root, _ = world
    ds = common(root) + ["--device-sampling", "--accumulation-steps", 2, "--random-crop", "--frames", 40]
    full = run(root, *ds, "--out", root / "ds.gguf", "--checkpoint-every", 2)
    assert full.returncode == 0, full.stderr
    resumed = run(root, *ds, "--out", root / "ds-resumed.gguf", "--resume", root / "ds.step-2.gguf.state")
    assert resumed.returncode == 0, resumed.stderr
    assert (root / "ds.gguf").read_bytes() == (root / "ds-resumed.gguf").read_bytes()
    host = run(root, *[a for a in ds if a != "--device-sampling"], "--out", root / "ds-host.gguf")
    assert host.returncode == 0, host.stderr
    assert (root / "ds.gguf").read_bytes() != (root / "ds-host.gguf").read_bytes()
    # the state records the sampling mode: a host-sampling resume of it is refused
    mixed = run(root, *[a for a in ds if a != "--device-sampling"], "--out", root / "ds-mixed.gguf", "--resume",
                root / "ds.step-2.gguf.state")
    assert mixed.returncode != 0 and not (root / "ds-mixed.gguf").exists()
    bridge = run(root, *common(root, "bridge_train", "bridge_validation"), "--objective", "edit-bridge",
                 "--device-sampling", "--out", root / "ds-bridge.gguf")
    assert bridge.returncode != 0 and not (root / "ds-bridge.gguf").exists()
