"""mg-train on the GPU: the reference CLI test's contract (tests/mg_train_cli_test.py of the reference:
checkpoints leave training unchanged, training-only caption pools, exact resume with accumulation /
warm-up / decay / crops / FFN targets, evaluation-only scoring, full-sequence and LoRA variants,
rejected settings) on an LM our kernels run, plus the printed losses against a replay of the same
draws through the CPU oracle."""
import json
import os
import re
import subprocess

import numpy as np
import pytest

import trainer_fixtures as TF

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "audiocraft.cpp_b200", "bin", "mg-train")
LOSS_REL = 1e-3


@pytest.fixture(scope="module")
def world(tmp_path_factory):
    if not os.path.exists(EXE):
        pytest.skip("mg-train is not built")
    root = tmp_path_factory.mktemp("mgtrain")
    lm = TF.TinyLm()
    lm.write(root / "base.gguf")
    TF.write_mg_caches(root / "train", lm, 2, 24, seed=5)
    TF.write_mg_caches(root / "validation", lm, 2, 20, seed=6, caption="HELD OUT CAPTION")
    return root, lm


def run(root, *args):
    return subprocess.run([EXE, "--lm", str(root / "base.gguf"), *map(str, args)], capture_output=True, text=True,
                          timeout=600)


def common(root):
    return ["--cache", root / "train", "--validation", root / "validation", "--frames", 20, "--prefix-frames", 3,
            "--steps", 4, "--rank", 4, "--first-layer", 0]


def test_losses_follow_the_oracle_replay(world):
    root, lm = world
    out = root / "parity.gguf"
    r = run(root, *common(root), "--out", out, "--steps", 3, "--adapter-type", "lora", "--alpha", 8,
            "--accumulation-steps", 2, "--random-crop", "--train-ffn", "--cfg-dropout", 0.3, "--lr", 2e-3,
            "--warmup-steps", 2, "--weight-decay", 0.01, "--seed", 77, "--checkpoint-every", 0)
    assert r.returncode == 0, r.stderr
    rep = TF.MgTrainReplay(lm, TF.read_mg_caches(root / "train"), TF.read_mg_caches(root / "validation"), 20, 3, 4,
                           8.0, 0, 77, 0x7F, accumulation=2, dropout=0.3, random_crop=True, lr=2e-3, warmup=2,
                           decay=0.01)
    want = rep.train(3)
    before = float(re.search(r"probe before ([-0-9.]+)", r.stderr).group(1))
    steps = [float(x) for x in re.findall(r"\] step \d+/\d+ windows \d+ lr \S+ loss ([-0-9.]+)", r.stderr)]
    after = float(re.search(r"fixed probe after ([-0-9.]+)", r.stderr).group(1))
    assert len(steps) == 3
    for got, ref in [(before, want["before"])] + list(zip(steps, want["steps"])) + [(after, want["after"])]:
        assert abs(got - ref) <= LOSS_REL * abs(ref), (got, ref, r.stderr)
    params, meta = TF.read_adapter(out)
    got = np.concatenate([params[name] for name, _, _ in rep.layout])
    assert np.linalg.norm(got - rep.params) <= 5e-3 * np.linalg.norm(rep.params)  # AdamW: see the mf-train test
    assert meta["ac.lora.training_objective"] == "continuation-cross-entropy"
    assert meta["ac.lora.training_frames"] == 20 and meta["ac.lora.prefix_frames"] == 3


def test_checkpoints_pools_and_base(world):
    root, _ = world
    base = (root / "base.gguf").read_bytes()
    for name, extra in [("plain", ["--checkpoint-every", 0]), ("checkpointed", ["--checkpoint-every", 2])]:
        r = run(root, *common(root), "--out", root / f"{name}.gguf", *extra)
        assert r.returncode == 0, r.stderr
        pool = json.loads((root / f"{name}.prompts.json").read_text(encoding="utf-8"))
        assert pool["dice"]["instrumental"] == ["glitch hop, 92 bpm, D minor"]
        assert pool["source"]["files"] == 2
    assert (root / "checkpointed.step-2.prompts.json").exists()
    assert (root / "plain.gguf").read_bytes() == (root / "checkpointed.gguf").read_bytes()
    assert (root / "base.gguf").read_bytes() == base
    params, meta = TF.read_adapter(root / "plain.gguf")
    assert meta["ac.lora.type"] == "dora-rows" and len(params) == 2 * 5 * 3


def test_exact_resume_and_adapter_scoring(world):
    root, _ = world
    controls = ["--accumulation-steps", 3, "--warmup-steps", 3, "--lr-schedule", "inverse", "--weight-decay", 0.01,
                "--beta2", 0.95, "--random-crop", "--train-ffn"]
    cropped = common(root) + ["--frames", 16] + controls
    full = run(root, *cropped, "--out", root / "controls.gguf", "--checkpoint-every", 2)
    assert full.returncode == 0, full.stderr
    resumed = run(root, *cropped, "--out", root / "resumed.gguf", "--checkpoint-every", 0, "--resume",
                  root / "controls.step-2.gguf.state")
    assert resumed.returncode == 0, resumed.stderr
    assert (root / "controls.gguf").read_bytes() == (root / "resumed.gguf").read_bytes()
    assert (root / "controls.gguf.state").read_bytes() == (root / "resumed.gguf.state").read_bytes()
    scored = run(root, *cropped, "--evaluate-adapter", root / "controls.gguf", "--eval-unconditional")
    assert scored.returncode == 0 and "[eval]" in scored.stderr, scored.stderr
    params, _ = TF.read_adapter(root / "controls.gguf")
    assert any(".ff.0." in n for n in params)
    changed = run(root, *cropped, "--out", root / "bad-resume.gguf", "--resume", root / "controls.step-2.gguf.state",
                  "--lr", 2e-4)
    assert changed.returncode != 0 and not (root / "bad-resume.gguf").exists()


def test_full_sequence_lora_and_evaluation(world):
    root, _ = world
    full = [a for a in common(root)]
    i = full.index("--prefix-frames")
    del full[i:i + 2]
    r = run(root, *full, "--out", root / "full.gguf", "--checkpoint-every", 0)
    assert r.returncode == 0, r.stderr
    _, meta = TF.read_adapter(root / "full.gguf")
    assert meta["ac.lora.prefix_frames"] == 0 and meta["ac.lora.training_objective"] == "generation-cross-entropy"
    r = run(root, *full, "--out", root / "lora.gguf", "--adapter-type", "lora", "--checkpoint-every", 0)
    assert r.returncode == 0, r.stderr
    params, meta = TF.read_adapter(root / "lora.gguf")
    assert meta["ac.lora.type"] == "lora" and len(params) == 2 * 5 * 2
    r = run(root, *full, "--evaluate-adapter", root / "full.gguf", "--eval-samples", 0)
    assert r.returncode == 0 and "[eval]" in r.stderr, r.stderr
    r = run(root, *full, "--evaluate-adapter", root / "lora.gguf")  # dora-rows context, lora adapter
    assert r.returncode != 0 and "mismatch" in r.stderr


@pytest.mark.parametrize("extra", [["--prefix-frames", 20], ["--adapter-type", "invalid"], ["--cfg-dropout", "nan"],
                                   ["--lr", "inf"], ["--alpha", -2], ["--first-layer", -2]])
def test_rejected_settings(world, extra):
    root, _ = world
    r = run(root, *common(root), "--out", root / "invalid.gguf", *extra)
    assert r.returncode != 0 and not (root / "invalid.gguf").exists()


def test_overlap_and_existing_output(world):
    root, _ = world
    r = run(root, *common(root), "--out", root / "overlap.gguf", "--validation", root / "train")
    assert r.returncode != 0 and "overlap" in r.stderr
    (root / "exists.gguf").write_bytes(b"x")
    r = run(root, *common(root), "--out", root / "exists.gguf")
    assert r.returncode != 0
