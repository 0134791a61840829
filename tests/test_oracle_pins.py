"""Pins the CPU oracle to the reference's own kernel self-checks (kernels/src/lib.rs:513-712):
the oracle, run on the replayed input stream, must reproduce tests/golden/reference_checks.npz
(the restated reference formulas in float64, made by tests/golden/make_golden.py) within the
reference's tolerances, and the reference's argmax known answer exactly."""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
import refchecks as rc

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "reference_checks.npz")


@pytest.fixture(scope="module")
def cases():
    return rc.replay()


def test_rng_stream_matches_reference_port():
    r = oracle.Rng(rc.SEED)
    assert np.array_equal(r.u32(16), GOLDEN["rng_u32_head"])
    r = oracle.Rng(rc.SEED)
    assert np.array_equal(r.f32(16), GOLDEN["rng_f32_head"])


def test_replay_consumes_the_whole_stream(cases):
    assert cases["rng_state_end"] == int(GOLDEN["rng_state_end"][0])


@pytest.mark.parametrize("i", range(len(rc.GEMV_ORDER)))
def test_gemv_checks(cases, i):
    c = cases["gemv"][i]
    out_rows = c.rows // 2 if c.epilogue == "swiglu" else c.rows
    y = c.y0.copy() if c.epilogue == "accumulate" else np.zeros(out_rows, np.float32)
    oracle.gemv("q4", c.w, c.s, c.z, c.rows, c.k, c.x, y, rc.EPI[c.epilogue])
    assert rc.rel_err(y, GOLDEN[c.name]) < rc.TOL_GEMV


@pytest.mark.parametrize("i", range(3))
def test_gemm_checks_as_per_token_gemv(cases, i):
    c = cases["gemm"][i]
    out_rows = c.rows // 2 if c.epilogue == "swiglu" else c.rows
    got = []
    for t in range(11):
        y = c.y0[t].copy() if c.epilogue == "accumulate" else np.zeros(out_rows, np.float32)
        oracle.gemv("q4", c.w, c.s, c.z, c.rows, c.k, c.x[t], y, rc.EPI[c.epilogue])
        got.append(y)
    assert rc.rel_err(np.stack(got), GOLDEN[c.name]) < rc.TOL_GEMV


def test_gdn_check(cases):
    g = cases["gdn"]
    conv = g["conv0"].copy()
    state = g["state0"].copy()
    out = oracle.gdn_step(g["proj"], conv, g["conv_w"], state, g["params"])
    assert rc.rel_err(out, GOLDEN["gdn_output"]) < rc.TOL_GDN_OUT
    assert rc.rel_err(state[::61], GOLDEN["gdn_state_sample"]) < rc.TOL_GDN_STATE
    sums = state.astype(np.float64).reshape(16, -1).sum(axis=1)
    assert np.allclose(sums, GOLDEN["gdn_state_head_sums"], rtol=1e-4, atol=1e-3)
    # conv windows shift: newest input last
    assert np.array_equal(conv[2::3], g["proj"][:6144])
    assert np.array_equal(conv[1::3], g["conv0"][2::3])


def test_attention_check(cases):
    a = cases["attention"]
    kc, vc = a["kc"].copy(), a["vc"].copy()
    rope = oracle.rope_table(1e7)
    out = oracle.attention_step(a["proj"], kc, vc, a["pos"], a["norms"], rope, kv_f16=False)
    assert rc.rel_err(out, GOLDEN["attention"]) < rc.TOL_ATTN


def test_attention_f16_cache_stays_close(cases):
    a = cases["attention"]
    rope = oracle.rope_table(1e7)
    f32 = oracle.attention_step(a["proj"], a["kc"].copy(), a["vc"].copy(), a["pos"], a["norms"], rope, False)
    f16 = oracle.attention_step(a["proj"], a["kc"].copy(), a["vc"].copy(), a["pos"], a["norms"], rope, True)
    assert rc.rel_err(f16, f32) < 2e-3


def test_embed_and_argmax_known_answer(cases):
    e = cases["embed"]
    row = oracle.dequant_rows("q4", e["w"], e["s"], e["z"], 300, 1024, 7, 1)[0]
    assert rc.rel_err(row, GOLDEN["embed"]) < rc.TOL_EMBED
    assert np.array_equal(row, GOLDEN["embed"])  # the unpack is exact
    tok = oracle.argmax(e["logits"])
    assert [tok, 41 + 1] == list(GOLDEN["argmax_tok"]) == [123457, 42]


def test_f16_to_f32_port_matches_ieee_for_finite_values():
    bits = np.arange(0, 1 << 16, 97, dtype=np.uint32)
    for b in bits:
        if (b >> 10) & 0x1F == 31:
            continue
        want = np.array([b], np.uint16).view(np.float16).astype(np.float32)[0]
        assert oracle.f16_to_f32_ref(int(b)) == want


def test_argmax_ties_take_lowest_index():
    x = np.zeros(1000, np.float32)
    x[[17, 400, 999]] = 3.0
    assert oracle.argmax(x) == 17
    x[5] = np.nan
    assert oracle.argmax(x) == 17
