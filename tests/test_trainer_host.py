"""Host side of the trainer front ends (audiocraft.cpp_b200/trainer), on the CPU.

A small C++ program built from the trainer sources prints what they produce: the C++ standard
library draws the CLIs make (pinned here against tests/stdrng.py, which the GPU tests use to replay
mf-train for the oracle), GGUF files (cross-checked with the gguf package), the exact-resume state
file, the caption pool and the learning-rate schedule (against the oracle's restatement of
src/ac/train_controls.h:53-58).  The CLIs' argument checks run before any device call, so they are
exercised here too.
"""
import json
import os
import struct
import subprocess

import numpy as np
import pytest

import stdrng as R

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "audiocraft.cpp_b200")
TRAINER = os.path.join(PKG, "trainer")

PROGRAM = r"""
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <iostream>
#include <random>
#include <string>
#include <vector>
#include "gguf_file.h"
#include "train_host.h"
using namespace actf;
int main(int argc, char** argv) {
    const std::string mode = argv[1];
    if (mode == "draws") {
        std::mt19937 g(1234);
        for (int i = 0; i < 700; ++i) std::printf("raw %u\n", (unsigned)g());
        std::mt19937 h(77);
        for (int i = 0; i < 50; ++i) std::printf("canon %a\n", std::generate_canonical<float, 24>(h));
        std::normal_distribution<float> n01;
        for (int i = 0; i < 301; ++i) std::printf("normal %a\n", n01(h));
        std::normal_distribution<float> n2(0.3f, 2.0f);
        for (int i = 0; i < 51; ++i) std::printf("normal2 %a\n", n2(h));
        for (int b : {1, 2, 7, 100, 1000003})
            for (int i = 0; i < 20; ++i) std::printf("int %d %d\n", b, std::uniform_int_distribution<int>(0, b)(h));
        for (int n = 1; n <= 9; ++n) {
            std::vector<size_t> v(n);
            for (int i = 0; i < n; ++i) v[i] = i;
            std::shuffle(v.begin(), v.end(), h);
            std::printf("shuffle %d", n);
            for (auto x : v) std::printf(" %zu", x);
            std::printf("\n");
        }
        MfTimeSampler uni("uniform", 0, 1), logit("logit-normal", 0.4f, 1.3f);
        for (int i = 0; i < 40; ++i) std::printf("tu %a\n", uni.sample(h));
        for (int i = 0; i < 40; ++i) std::printf("tl %a\n", logit.sample(h));
        std::printf("next %u\n", (unsigned)h());
        return 0;
    }
    if (mode == "write_gguf") {
        GgufWriter w;
        w.add_string("general.architecture", "ac-melodyflow-lora");
        w.add_u32("ac.lora.rank", 4);
        w.add_f32("ac.lora.alpha", 8.0f);
        w.add_bool("ac.flag", true);
        w.add_string("ac.lora.type", "dora-rows");
        w.add_u32("ac.lora.rank", 5);  // a key set twice keeps its place
        std::vector<float> a(3 * 40), b(7);
        for (size_t i = 0; i < a.size(); ++i) a[i] = 0.5f * (float)i - 3.0f;
        for (size_t i = 0; i < b.size(); ++i) b[i] = 1.0f / (float)(i + 1);
        w.add_f32_tensor("dit.0.self.qkv.weight.lora_A", {40, 3}, a.data());
        w.add_f32_tensor("dit.0.self.qkv.weight.magnitude", {7, 1}, b.data());
        w.write(argv[2]);
        try {
            w.write(argv[2]);
            std::printf("overwrote\n");
        } catch (const std::exception& e) {
            std::printf("refused %s\n", e.what());
        }
        return 0;
    }
    if (mode == "read_gguf") {
        GgufReader r(argv[2]);
        std::printf("name %s\n", r.string("general.name").c_str());
        std::printf("dim %u\n", r.u32("ac.dit.dim"));
        std::printf("eps %a\n", r.f32("ac.dit.norm_eps"));
        std::printf("zero %d\n", (int)r.boolean("ac.dit.add_zero_attn"));
        for (const auto& t : r.tensors()) {
            std::printf("tensor %s %u %lld %lld %zu", t.name.c_str(), t.type, (long long)t.ne[0], (long long)t.ne[1],
                        t.bytes);
            double s = 0;
            if (t.type == GT_F32)
                for (int64_t i = 0; i < t.nelements(); ++i) s += reinterpret_cast<const float*>(t.data)[i] * (i + 1);
            std::printf(" %.9g\n", s);
        }
        try {
            r.u32("general.name");
        } catch (const std::exception& e) {
            std::printf("typed %s\n", e.what());
        }
        return 0;
    }
    if (mode == "state") {
        std::vector<HostParam> ps(2);
        ps[0].name = "dit.0.self.qkv.weight.lora_A";
        ps[1].name = "dit.0.self.qkv.weight.lora_B";
        for (int j = 0; j < 2; ++j)
            for (int i = 0; i < 5 + j; ++i) {
                ps[j].value.push_back(std::nextafter(0.1f * (i + 1), 1.0f) * (j ? -1 : 1));
                ps[j].m.push_back(1e-7f * (float)i);
                ps[j].v.push_back(3.0e-12f * (float)(i + j));
            }
        std::mt19937 rng(99);
        for (int i = 0; i < 1000; ++i) rng();
        std::vector<size_t> order{2, 0, 3, 1};
        int step = 7;
        size_t seen = 21;
        train_state(argv[2], false, "sig|1", ps, step, seen, rng, order);
        auto ps2 = ps;
        for (auto& p : ps2)
            for (auto* v : {&p.value, &p.m, &p.v}) std::fill(v->begin(), v->end(), 0.f);
        std::mt19937 rng2(1);
        std::vector<size_t> order2(4);
        int step2 = 0;
        size_t seen2 = 0;
        for (size_t i = 0; i < 4; ++i) order2[i] = i;
        train_state(argv[2], true, "sig|1", ps2, step2, seen2, rng2, order2);
        bool same = step2 == step && seen2 == seen && rng2 == rng && order2 == order;
        for (int j = 0; j < 2; ++j) same = same && ps2[j].value == ps[j].value && ps2[j].m == ps[j].m && ps2[j].v == ps[j].v;
        std::printf("roundtrip %d\n", (int)same);
        try {
            train_state(argv[2], true, "sig|2", ps2, step2, seen2, rng2, order2);
        } catch (const std::exception& e) {
            std::printf("mismatch %s\n", e.what());
        }
        try {
            train_state(argv[2], false, "sig|1", ps, step, seen, rng, order);
        } catch (const std::exception& e) {
            std::printf("exists %s\n", e.what());
        }
        return 0;
    }
    if (mode == "pool") {
        write_prompt_pool(argv[2], "/x/y/adapter.gguf",
                          {"calm piano", "", "calm piano", "caf\xc3\xa9 \"jazz\"\n", "\xf0\x9f\x8e\xb5 drums"}, 3);
        for (auto c : read_prompt_pool(argv[2])) {
            for (size_t i; (i = c.find('\n')) != std::string::npos;) c.replace(i, 1, "<NL>");
            std::printf("caption [%s]\n", c.c_str());
        }
        std::printf("path %s\n", prompt_pool_path("/a/b/c.step-2.gguf").c_str());
        return 0;
    }
    if (mode == "lora") {
        GgufReader base(argv[2]), adapter(argv[3]);
        try {
            const auto m = load_lora(base, adapter, std::stof(argv[5]), argv[4]);
            std::printf("ok %zu %a %d\n", m.size(), m[0].scale, (int)(m[0].magnitude != nullptr));
        } catch (const std::exception& e) {
            std::printf("error %s\n", e.what());
        }
        return 0;
    }
    if (mode == "rate") {
        for (const char* sched : {"constant", "inverse"})
            for (int warm : {0, 3, 50}) {
                TrainControls c;
                c.schedule = sched;
                c.warmup = warm;
                for (int step : {1, 2, 3, 4, 10, 1000, 250000}) std::printf("rate %s %d %d %a\n", sched, warm, step, c.rate(3e-4f, step));
            }
        TrainControls c;
        std::printf("sig %s\n", c.signature(1e-4f).c_str());
        std::printf("key %s\n", train_key(50, 8, 8.0f, 0.1f, 1234u, std::string("flow-matching"), 0.3f).c_str());
        return 0;
    }
    return 2;
}
"""


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    import subprocess as sp
    d = tmp_path_factory.mktemp("trainer_host")
    src = d / "harness.cpp"
    src.write_text(PROGRAM)
    exe = d / "harness"
    lib = os.path.join(PKG, "libactrain.so")
    if not os.path.exists(lib):
        pytest.skip("libactrain.so is not built")
    sp.run(["g++", "-std=c++17", "-O2", "-I" + TRAINER, "-I" + os.path.join(ROOT, "include"), str(src),
            os.path.join(TRAINER, "gguf_file.cpp"), os.path.join(TRAINER, "train_host.cpp"), "-o", str(exe),
            "-L" + PKG, "-lactrain", "-Wl,-rpath," + PKG], check=True)

    def run(*args):
        return sp.run([str(exe), *map(str, args)], capture_output=True, text=True, check=True, timeout=60).stdout

    run.dir = d
    return run


def _f(hexstr):
    return np.float32(float.fromhex(hexstr))


def test_stdlib_draws_match_the_python_replay(harness):
    lines = [l.split() for l in harness("draws").splitlines()]
    by = {}
    for l in lines:
        by.setdefault(l[0], []).append(l[1:])
    g = R.MT19937(1234)
    assert [int(x[0]) for x in by["raw"]] == [g() for _ in range(700)]
    h = R.MT19937(77)
    assert [_f(x[0]) for x in by["canon"]] == [R.canonical(h) for _ in range(50)]
    n01 = R.Normal()
    got = [_f(x[0]) for x in by["normal"]]
    assert got == [n01(h) for _ in range(301)]
    n2 = R.Normal(0.3, 2.0)
    assert [_f(x[0]) for x in by["normal2"]] == [n2(h) for _ in range(51)]
    assert [(int(b), int(v)) for b, v in by["int"]] == [(b, R.uniform_int(h, 0, b)) for b in (1, 2, 7, 100, 1000003)
                                                       for _ in range(20)]
    for x in by["shuffle"]:
        n = int(x[0])
        v = list(range(n))
        R.shuffle(v, h)
        assert [int(y) for y in x[1:]] == v, n
    assert [_f(x[0]) for x in by["tu"]] == [R.time_sample(h) for _ in range(40)]
    tl = [_f(x[0]) for x in by["tl"]]
    assert tl == [R.time_sample(h, "logit-normal", 0.4, 1.3) for _ in range(40)]
    assert all(1e-6 <= t <= 1 - 1e-6 for t in tl)
    assert int(by["next"][0][0]) == h()


def test_gguf_writer_is_read_by_the_gguf_package(harness):
    gguf = pytest.importorskip("gguf")
    path = harness.dir / "w.gguf"
    if path.exists():
        path.unlink()
    out = harness("write_gguf", path)
    assert "refused [gguf] refusing to overwrite" in out
    r = gguf.GGUFReader(str(path))
    kv = {f.name: f for f in r.fields.values()}
    assert kv["general.architecture"].contents() == "ac-melodyflow-lora"
    assert kv["ac.lora.rank"].contents() == 5 and kv["ac.lora.alpha"].contents() == 8.0
    assert kv["ac.flag"].contents() is True and kv["ac.lora.type"].contents() == "dora-rows"
    names = [f.name for f in r.fields.values() if not f.name.startswith("GGUF.")]
    assert names == ["general.architecture", "ac.lora.rank", "ac.lora.alpha", "ac.flag", "ac.lora.type"]
    t = {x.name: x for x in r.tensors}
    a = t["dit.0.self.qkv.weight.lora_A"]
    assert list(a.shape) == [40, 3] and a.tensor_type == gguf.GGMLQuantizationType.F32
    np.testing.assert_array_equal(np.asarray(a.data).ravel(), 0.5 * np.arange(120, dtype=np.float32) - 3.0)
    m = t["dit.0.self.qkv.weight.magnitude"]
    assert list(m.shape) == [7]  # ggml's n_dims: trailing unit axes are dropped
    np.testing.assert_array_equal(np.asarray(m.data).ravel(), (1.0 / np.arange(1, 8)).astype(np.float32))
    assert all(x.data_offset % 32 == 0 for x in r.tensors)


def test_gguf_reader_reads_the_gguf_package(harness, tmp_path):
    gguf = pytest.importorskip("gguf")
    path = tmp_path / "m.gguf"
    w = gguf.GGUFWriter(str(path), "audiocraft")
    w.add_string("general.name", "tiny model")
    w.add_uint32("ac.dit.dim", 128)
    w.add_float32("ac.dit.norm_eps", 1e-5)
    w.add_bool("ac.dit.add_zero_attn", True)
    w.add_array("ac.list", [1, 2, 3])
    x = np.arange(24, dtype=np.float32).reshape(4, 6)
    w.add_tensor("dit.x", x)
    h = (np.arange(64, dtype=np.float32) / 7).astype(np.float16).reshape(2, 32)
    w.add_tensor("dit.h", h)
    w.add_tensor("dit.q", np.arange(34 * 2, dtype=np.uint8).reshape(2, 34), raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    out = harness("read_gguf", path).splitlines()
    assert out[0] == "name tiny model" and out[1] == "dim 128"
    assert _f(out[2].split()[1]) == np.float32(1e-5) and out[3] == "zero 1"
    rows = {l.split()[1]: l.split()[2:] for l in out if l.startswith("tensor ")}
    assert rows["dit.x"][:4] == ["0", "6", "4", "96"]
    assert float(rows["dit.x"][4]) == float((x.ravel().astype(np.float64) * np.arange(1, 25)).sum())
    assert rows["dit.h"][:4] == ["1", "32", "2", "128"]
    assert rows["dit.q"][:4] == ["8", "32", "2", "68"]  # two rows of one 34-byte block
    assert any(l.startswith("typed [gguf] general.name is string") for l in out)


def test_resume_state_round_trips_exactly(harness):
    path = harness.dir / "s.state"
    if path.exists():
        path.unlink()
    out = harness("state", path)
    assert "roundtrip 1" in out
    assert "mismatch trainer state configuration/data mismatch" in out
    assert "exists trainer state already exists" in out
    text = path.read_text().split("\n")
    assert text[0] == '"ac-trainer-state-v1"' and text[1] == '"sig|1"' and text[2] == "7" and text[3] == "21"


def test_prompt_pool_round_trips_and_escapes(harness):
    path = harness.dir / "p.prompts.json"
    if path.exists():
        path.unlink()
    out = harness("pool", path)
    caps = [l[len("caption ["):-1] for l in out.split("\n") if l.startswith("caption [")]
    assert caps == ["calm piano", "café \"jazz\"<NL>", "\U0001F3B5 drums"]
    assert "path /a/b/c.step-2.prompts.json" in out
    doc = json.loads(path.read_text())
    assert doc["version"] == 1 and doc["source"] == {"lora": "adapter.gguf", "files": 3, "unique_prompts": 3}
    assert doc["dice"]["instrumental"] == ["calm piano", "café \"jazz\"\n", "\U0001F3B5 drums"]
    assert path.read_text().isascii()  # non-ASCII written as \\u escapes


def test_rate_schedule_matches_the_oracle(harness):
    import oracle as O
    lib = O.lib()
    for l in harness("rate").splitlines():
        if not l.startswith("rate "):
            continue
        _, sched, warm, step, v = l.split()
        want = lib.ora_rate(np.float32(3e-4), int(step), int(warm), int(sched == "inverse"))
        assert _f(v) == np.float32(want), l
    out = harness("rate")
    assert "sig 1 0 0.899999976 0.999000013 9.99999994e-09 0 1 constant 0 0 9.99999975e-05" in out
    assert "key 50|8|8|0.100000001|1234|flow-matching|0.300000012|" in out


BAD_FLAGS = [["--accumulation-steps", "0"], ["--warmup-steps", "-1"], ["--beta2", "1"], ["--weight-decay", "nan"],
             ["--lr-schedule", "bogus"], ["--adapter-type", "dora-cols"], ["--t-sampling", "unknown"],
             ["--t-std", "0"], ["--t-mean", "nan"], ["--eval-draws", "0"], ["--frames", "751"],
             ["--objective", "bogus"], ["--device", "cpu"], ["--bogus-flag"]]


@pytest.mark.parametrize("extra", BAD_FLAGS, ids=[" ".join(e) for e in BAD_FLAGS])
def test_cli_rejects_bad_settings_before_any_device_work(extra, tmp_path):
    exe = os.path.join(PKG, "bin", "mf-train")
    if not os.path.exists(exe):
        pytest.skip("mf-train is not built")
    out = tmp_path / "bad.gguf"
    r = subprocess.run([exe, "--dit", str(tmp_path / "missing.gguf"), "--cache", str(tmp_path), "--out", str(out)] + extra,
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "error:" in r.stderr and not out.exists(), r.stderr


def test_cli_usage_without_required_paths():
    exe = os.path.join(PKG, "bin", "mf-train")
    if not os.path.exists(exe):
        pytest.skip("mf-train is not built")
    r = subprocess.run([exe, "--steps", "3"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "usage: mf-train" in r.stderr


def _lora_files(tmp_path, kind="lora", **bad):
    """A tiny DiT base and an adapter for two projections, with one defect from `bad`."""
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(0)
    base = {"dit.0.self.qkv.weight": rng.standard_normal((24, 8)).astype(np.float32),
            "dit.1.ff.0.weight": rng.standard_normal((16, 8)).astype(np.float32)}
    w = gguf.GGUFWriter(str(tmp_path / "base.gguf"), "audiocraft")
    w.add_string("general.name", "tiny")
    for k, v in base.items():
        w.add_tensor(k, v)
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()
    r = 2
    t = {}
    for stem, W in base.items():
        t[stem + ".lora_A"] = rng.standard_normal((r, W.shape[1])).astype(np.float32)
        t[stem + ".lora_B"] = rng.standard_normal((W.shape[0], r)).astype(np.float32)
        if kind == "dora-rows":
            t[stem + ".magnitude"] = np.abs(rng.standard_normal(W.shape[0])).astype(np.float32)
    if bad.get("shape"):
        t["dit.1.ff.0.weight.lora_B"] = np.zeros((15, r), np.float32)
    if bad.get("missing"):
        del t["dit.1.ff.0.weight.lora_B"]
    if bad.get("extra"):
        t["dit.1.ff.0.weight.extra"] = np.zeros(3, np.float32)
    if bad.get("nan"):
        t["dit.0.self.qkv.weight.lora_A"][0, 0] = np.nan
    if bad.get("target"):
        base_name = "dit.0.self.qkv.weight"
        t = {k.replace(base_name, "dit.0.norm1.weight"): v for k, v in t.items()}
    arch = bad.get("arch", "ac-melodyflow-lora")
    w = gguf.GGUFWriter(str(tmp_path / "a.gguf"), arch)
    w.add_uint32("ac.lora.version", 1)
    w.add_uint32("ac.lora.rank", r)
    w.add_float32("ac.lora.alpha", 4.0)
    w.add_string("ac.lora.type", kind)
    w.add_string("ac.lora.base_name", bad.get("base_name", "tiny"))
    for k, v in t.items():
        w.add_tensor(k, v)
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()
    return tmp_path / "base.gguf", tmp_path / "a.gguf"


@pytest.mark.parametrize("kind", ["lora", "dora-rows"])
def test_adapter_loader_accepts_a_trained_adapter(harness, tmp_path, kind):
    base, ad = _lora_files(tmp_path, kind)
    out = harness("lora", base, ad, "dit", "0.5").split()
    assert out[0] == "ok" and out[1] == "2" and out[3] == ("1" if kind == "dora-rows" else "0")
    # load_lora: LoRA folds the strength into the scale, DoRA keeps it apart (src/ac/lora.h:141)
    assert _f(out[2]) == np.float32(np.float32(0.5 if kind == "lora" else 1.0) * np.float32(4.0) / np.float32(2))


@pytest.mark.parametrize("defect,message", [
    ({"shape": True}, "adapter shape mismatch: dit.1.ff.0.weight"),
    ({"missing": True}, "missing tensor dit.1.ff.0.weight.lora_B"),
    ({"extra": True}, "empty or incomplete adapter"),
    ({"nan": True}, "nonfinite adapter tensor"),
    ({"base_name": "other"}, "adapter base model name does not match"),
    ({"arch": "ac-musicgen-lora"}, "not a MelodyFlow adapter"),
], ids=["shape", "missing", "extra", "nan", "base_name", "arch"])
def test_adapter_loader_rejects_what_the_reference_rejects(harness, tmp_path, defect, message):
    base, ad = _lora_files(tmp_path, **defect)
    out = harness("lora", base, ad, "dit", "1")
    assert out.startswith("error ") and message in out, out


def test_adapter_loader_rejects_unsupported_targets(harness, tmp_path):
    gguf = pytest.importorskip("gguf")
    base, ad = _lora_files(tmp_path, target=True)
    out = harness("lora", base, ad, "dit", "1")
    assert out.startswith("error ")  # the base has no dit.0.norm1.weight, or the target is refused


MG_BAD = [["--accumulation-steps", "0"], ["--lr-schedule", "bogus"], ["--cfg-dropout", "nan"], ["--lr", "inf"],
          ["--steps", "0"], ["--device", "cpu"], ["--bogus-flag"]]


@pytest.mark.parametrize("extra", MG_BAD, ids=[" ".join(e) for e in MG_BAD])
def test_mg_cli_rejects_bad_settings_before_any_device_work(extra, tmp_path):
    exe = os.path.join(PKG, "bin", "mg-train")
    if not os.path.exists(exe):
        pytest.skip("mg-train is not built")
    out = tmp_path / "bad.gguf"
    r = subprocess.run([exe, "--lm", str(tmp_path / "missing.gguf"), "--cache", str(tmp_path), "--out", str(out)] + extra,
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "error:" in r.stderr and not out.exists(), r.stderr
