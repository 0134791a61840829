"""The weight-format converter (qne.convert) on the CPU: every matrix of the converted file,
decoded by the CPU oracle, against the source decoded the same way (bit-exact for q4 -> f16,
within half a quantization step for the int4 targets), the file conventions (256-byte alignment,
the tied embedding stored once, non-matrix tensors copied), byte-for-byte copies when the kind
does not change, and the decode step of a converted model against the source model's."""
import json
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle
from qne import convert, synth

VOCAB = 512


def mats(index_json, weights):
    """name -> (kind, rows, k, w, s, z) as numpy views of the weights."""
    idx = json.loads(index_json)
    out = {}
    for name, m in idx["matrices"].items():
        kind = m.get("kind", "q4")
        parts = {}
        for p, nbytes in convert.part_bytes(kind, m["rows"], m["k"]).items():
            t = idx["tensors"][f"{name}.{p}"]
            assert t["bytes"] == nbytes
            parts[p] = weights[t["offset"]:t["offset"] + nbytes]
        out[name] = (kind, m["rows"], m["k"], parts.get("w"), parts.get("s"), parts.get("z"))
    return out


def oracle_decode(kind, rows, k, w, s, z):
    return oracle.dequant_rows(kind, w, s, z, rows, k, 0, rows)


@pytest.fixture(scope="module")
def q4_model():
    return synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="q4", embed_kind="q4", seed=41)


@pytest.fixture(scope="module")
def f16_model():
    return synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="f16", seed=42)


def test_q4_to_f16_is_one_rounding_of_the_decoded_values(q4_model):
    idx, w = convert.convert(q4_model.index_json, q4_model.weights, "f16")
    src, dst = mats(q4_model.index_json, q4_model.weights), mats(idx, w)
    for name, (kind, rows, k, *parts) in src.items():
        assert kind == "q4" and dst[name][0] == "f16"
        want = oracle_decode(kind, rows, k, *parts).astype(np.float16)
        got = dst[name][3].view(np.float16).reshape(rows, k)
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), name


@pytest.mark.parametrize("target", ["q4", "q4g64"])
def test_f16_to_int4_decodes_within_half_a_step(f16_model, target):
    idx, w = convert.convert(f16_model.index_json, f16_model.weights, target, embed_kind="f16")
    src, dst = mats(f16_model.index_json, f16_model.weights), mats(idx, w)
    g = 32 if target == "q4" else 64
    for name, (kind, rows, k, sw, _, _) in src.items():
        x = sw.view(np.float16).reshape(rows, k).astype(np.float32)
        dkind, _, _, dw, ds, dz = dst[name]
        if name in ("embed", "lm_head"):
            assert dkind == "f16" and np.array_equal(dw, sw)  # same kind: copied
            continue
        assert dkind == target
        got = oracle_decode(target, rows, k, dw, ds, dz)
        step = ds.view(np.float16).astype(np.float32).reshape(rows, k // g)
        err = np.abs(got - x).reshape(rows, k // g, g).max(axis=-1)
        assert np.all(err <= 0.52 * step + 1e-12), (name, float((err / np.maximum(step, 1e-30)).max()))
        assert np.abs(got - x).mean() < 0.3 * step.mean()


def test_file_conventions_and_copies(f16_model):
    idx_s, w = convert.convert(f16_model.index_json, f16_model.weights, "f16")
    idx = json.loads(idx_s)
    src = json.loads(f16_model.index_json)
    assert idx["config"] == src["config"] and idx["format_version"] == 1
    for name, t in idx["tensors"].items():
        assert t["offset"] % 256 == 0 and t["offset"] + t["bytes"] <= w.size
        s = src["tensors"][name]
        assert np.array_equal(w[t["offset"]:t["offset"] + t["bytes"]],
                              f16_model.weights[s["offset"]:s["offset"] + s["bytes"]]), name
    assert idx["tensors"]["embed.w"]["offset"] == idx["tensors"]["lm_head.w"]["offset"]  # tied: stored once
    assert w.size <= f16_model.weights.size


def test_q4g64_to_q4g64_is_a_byte_copy():
    s = synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="q4g64", seed=43)
    idx_s, w = convert.convert(s.index_json, s.weights, "q4g64", embed_kind="f16")
    a, b = mats(s.index_json, s.weights), mats(idx_s, w)
    for name in a:
        for i in (3, 4, 5):
            assert (a[name][i] is None and b[name][i] is None) or np.array_equal(a[name][i], b[name][i])


def test_errors():
    s = synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="f16", seed=44)
    with pytest.raises(ValueError):
        convert.convert(s.index_json, s.weights, "q8")
    idx = json.loads(s.index_json)
    idx["tensors"]["layer0.down.w"]["bytes"] -= 2
    with pytest.raises(ValueError, match="invalid tensor size"):
        convert.convert(json.dumps(idx), s.weights, "q4g64")
    with pytest.raises(ValueError, match="does not fit"):
        convert.encode_rows("q4g64", np.full((1, 64), 1e6, np.float32))
    enc = convert.encode_rows("q4", np.zeros((2, 64), np.float32))  # an all-zero group decodes to zero
    dec = convert.decode_rows("q4", enc, 2, 64, 0, 2)
    assert np.array_equal(dec, np.zeros((2, 64), np.float32))


def test_converted_model_decodes_like_the_source(q4_model):
    """The decode step (CPU oracle) over the q4 model and over its f16 conversion: the only
    difference is one f16 rounding per weight."""
    idx, w = convert.convert(q4_model.index_json, q4_model.weights, "f16")
    a = oracle.OracleModel(q4_model.index_json, q4_model.weights, kv_f16=True)
    b = oracle.OracleModel(idx, w, kv_f16=True)
    prompt = synth.prompt_ids(6, 5, VOCAB)
    la, lb = a.prefill(prompt), b.prefill(prompt)
    assert np.abs(la - lb).max() <= 2e-2 * max(1.0, np.abs(la).max())
    assert oracle.argmax(la) == oracle.argmax(lb) or np.sort(la)[-1] - np.sort(la)[-2] < 4e-2
    a.close()
    b.close()


def test_command_line(tmp_path, f16_model):
    f16_model.save(tmp_path / "src")
    root = __import__("pathlib").Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "-m", "qne.convert", str(tmp_path / "src"), str(tmp_path / "out"),
                        "--kind", "q4g64", "--embed-kind", "f16"],
                       cwd=root / "qwen-native-engine_b200", capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    idx = json.loads((tmp_path / "out" / "index.json").read_text())
    w = np.fromfile(tmp_path / "out" / "weights.bin", np.uint8)
    assert idx["matrices"]["layer0.gate_up"]["kind"] == "q4g64" and idx["matrices"]["embed"]["kind"] == "f16"
    assert max(t["offset"] + t["bytes"] for t in idx["tensors"].values()) == w.size
    assert not (tmp_path / "out" / "weights.bin.tmp").exists()
