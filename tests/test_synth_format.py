"""The synthetic writer produces the converter's weights.bin / index.json format
(scripts/convert_weights.py:35-66): 256-byte aligned tensors, tied embedding stored once,
per-kind tensor sizes, the benchmark value distributions."""
import json

import numpy as np
import pytest

from qne import synth


@pytest.mark.parametrize("kind", ["f16", "q4", "q4g64"])
def test_layout(kind):
    s = synth.build(1024, 3584, layers=4, vocab=1000, kind=kind, seed=1)
    idx = json.loads(s.index_json)
    t = idx["tensors"]
    for name, e in t.items():
        assert e["offset"] % 256 == 0, name
        assert e["offset"] + e["bytes"] <= s.weights.nbytes
    assert t["embed.w"] == t["lm_head.w"]
    el = 8224 * 1024
    sizes = {"f16": {"w": el * 2}, "q4": {"w": el // 2, "s": el // 16, "z": el // 64},
             "q4g64": {"w": el // 2, "s": el // 32, "z": el // 32}}[kind]
    for part, n in sizes.items():
        assert t[f"layer0.mixer_in.{part}"]["bytes"] == n
    assert idx["matrices"]["layer3.mixer_in"]["rows"] == 5120
    assert idx["matrices"]["layer2.gate_up"]["rows"] == 2 * 3584


def test_values_follow_the_configs():
    s = synth.build(1024, 3584, layers=4, vocab=4096, kind="f16", seed=0)
    idx = json.loads(s.index_json)
    t = idx["tensors"]

    def arr(name, dt):
        e = t[name]
        return s.weights[e["offset"]:e["offset"] + e["bytes"]].view(dt)

    w = arr("layer1.gate_up.w", np.float16).astype(np.float32)
    assert abs(w.std() - 0.02) < 1e-3 and abs(w.mean()) < 1e-3
    assert np.all(arr("layer0.input_norm", np.float32) == 1)
    p = arr("layer0.gdn_params", np.float32)
    assert np.all(p[:16] == 0) and np.all(p[16:32] == -0.5) and np.all(p[32:] == 1)
    cw = arr("layer0.conv_w", np.float32)
    assert cw.min() >= -0.5 and cw.max() < 0.5
    q = synth.build(1024, 3584, layers=4, vocab=4096, kind="q4g64", seed=2)
    qt = json.loads(q.index_json)["tensors"]
    z = q.weights[qt["layer0.down.z"]["offset"]:][: qt["layer0.down.z"]["bytes"]].view(np.float16)
    assert np.all(z == 8)
    sc = q.weights[qt["layer0.down.s"]["offset"]:][: qt["layer0.down.s"]["bytes"]].view(np.float16).astype(np.float32)
    assert sc.min() >= 0 and 0.005 < sc.mean() < 0.012


def test_deterministic():
    a = synth.build(1024, 3584, layers=4, vocab=300, seed=7)
    b = synth.build(1024, 3584, layers=4, vocab=300, seed=7)
    c = synth.build(1024, 3584, layers=4, vocab=300, seed=8)
    assert np.array_equal(a.weights, b.weights)
    assert not np.array_equal(a.weights, c.weights)


def test_prompt_ids():
    p = synth.prompt_ids(128, 0)
    assert p.dtype == np.uint32 and p.max() < synth.VOCAB and len(set(p.tolist())) > 100
    assert np.array_equal(p, synth.prompt_ids(128, 0))
