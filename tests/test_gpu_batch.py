"""Batched decode (independent sequences, benchmark config 4) on the B200: the tensor-core GEMM
against the oracle GEMV per sequence, the whole batched step against one oracle model per
sequence, and page-table permutations that must not change a single bit."""
import numpy as np
import pytest
import torch

import qne
import refchecks as rc
from oracle import oracle
from qne import synth

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("impl", ["tcgen05", "mma_sync"])
@pytest.mark.parametrize("batch", [1, 3, 8, 13, 16, 17, 32, 33, 50, 64])
@pytest.mark.parametrize("epilogue,rows,k", [("store", 1024, 1024), ("accumulate", 1024, 3584), ("swiglu", 2 * 3584, 1024),
                                             ("store", 8224, 2048), ("store", 4099, 1024), ("accumulate", 2048, 6144),
                                             ("swiglu", 2 * 6144, 2048), ("store", 1000, 96), ("swiglu", 2 * 200, 4160),
                                             ("store", 40000, 1024)])  # > 2 waves of tiles: the 4-stage ring
def test_gemm_matches_gemv_per_sequence(cuda, impl, batch, epilogue, rows, k):
    if impl == "mma_sync" and batch > 32:
        pytest.skip("the mma.sync GEMM takes batch 1..32")
    rng = np.random.default_rng(batch * 7 + rows)
    w = (rng.standard_normal(rows * k) * 0.05).astype(np.float16)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal((batch, out_rows)).astype(np.float32)
    wd = dev(w)
    m = qne.matrix("f16", rows, k, wd)
    xd = dev(x)
    yd = dev(y0 if epilogue == "accumulate" else np.zeros((batch, out_rows), np.float32))
    qne.gemm(m, xd, batch, yd, epilogue, impl=impl)
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    for b in range(batch):
        want = y0[b].copy() if epilogue == "accumulate" else np.zeros(out_rows, np.float32)
        oracle.gemv("f16", w, None, None, rows, k, x[b], want, rc.EPI[epilogue])
        assert rc.rel_err(got[b], want) < 1e-4, b


def test_gemm_batch_limits(cuda):
    """Batches past a kernel's limit are rejected before anything runs: 64 rows on the tensor-core
    GEMM, 32 on the mma.sync one."""
    w = dev(np.zeros(256 * 64, np.float16))
    m = qne.matrix("f16", 256, 64, w)
    x = dev(np.zeros((65, 64), np.float32))
    y = dev(np.zeros((65, 256), np.float32))
    for impl, limit in (("tcgen05", 64), ("mma_sync", 32)):
        qne.gemm(m, x, limit, y, "store", impl=impl)
        with pytest.raises(qne.QneError) as e:
            qne.gemm(m, x, limit + 1, y, "store", impl=impl)
        assert e.value.name == "EINVAL" and f"1..{limit}" in str(e.value)
    torch.cuda.synchronize()


@pytest.fixture(scope="module")
def tiny(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=8192, kind="f16", seed=21)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    yield s, m
    m.close()


def test_batched_decode_matches_oracle_per_sequence(tiny):
    s, m = tiny
    B, L, steps = 5, 12, 16
    prompts = np.stack([synth.prompt_ids(L, 100 + b, 8192) for b in range(B)])
    bt = qne.Batch(m, B)
    for t in range(L):
        nxt, lg = bt.step(prompts[:, t], np.full(B, t), want_logits=True)
    ids = [nxt.copy()]
    cur = nxt.copy()
    step_logits = []
    for i in range(steps):
        cur, lg2 = bt.step(cur, np.full(B, L + i), want_logits=True)
        ids.append(cur.copy())
        step_logits.append(lg2.copy())
    ids = np.stack(ids, 1)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    for b in range(B):
        om.reset()
        want = om.prefill(prompts[b])
        err = np.abs(lg[b].astype(np.float64) - want).max()
        assert err <= 2e-2 and rc.rel_err(lg[b], want) <= 1e-3, (b, err)
        want_ids, margins = om.greedy(want, L, steps + 1)
        for i, (a, w_) in enumerate(zip(ids[b], want_ids)):
            if a != w_:
                assert margins[i] < 4e-2, (b, i, a, w_, margins[i])
                break
    om.close()
    bt.close()


@pytest.mark.parametrize("kind", ["q4", "q4g64"])
def test_int4_batched_decode_matches_oracle(cuda, kind):
    """int4 models (the reference converter's block-32 layout, with an int4 LM head; and group 64
    with an f16 LM head): every batched GEMM widens its nibbles to f16 in shared memory, so a step
    launches what an f16 step launches. Per-sequence logits against the oracle after the prompt,
    then greedy continuations."""
    s = synth.build(1024, 3584, layers=4, vocab=8192, kind=kind, embed_kind="q4" if kind == "q4" else "f16",
                    seed=24)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    B, L, steps = 3, 10, 8
    prompts = np.stack([synth.prompt_ids(L, 400 + b, 8192) for b in range(B)])
    bt = qne.Batch(m, B)
    for t in range(L):
        launches0 = qne.kernel_launches()
        nxt, lg = bt.step(prompts[:, t], np.full(B, t), want_logits=True)
        # no decode-to-f16 launches; the attention layers' merge writes the out-projection's planes
        assert qne.kernel_launches() - launches0 == 6 * m.layers + 3 - m.layers // 4
    ids = [nxt.copy()]
    cur = nxt.copy()
    for i in range(steps):
        cur = bt.step(cur, np.full(B, L + i))
        ids.append(cur.copy())
    ids = np.stack(ids, 1)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    for b in range(B):
        om.reset()
        want = om.prefill(prompts[b])
        err = np.abs(lg[b].astype(np.float64) - want).max()
        assert err <= 2e-2 and rc.rel_err(lg[b], want) <= 1e-3, (b, err)
        want_ids, margins = om.greedy(want, L, steps + 1)
        for i, (a, w_) in enumerate(zip(ids[b], want_ids)):
            if a != w_:
                assert margins[i] < 4e-2, (b, i, a, w_, margins[i])
                break
    om.close()
    bt.close()
    m.close()


def test_page_table_permutation_is_bit_exact(tiny):
    s, m = tiny
    B, L = 3, 40
    prompts = np.stack([synth.prompt_ids(L, 200 + b, 8192) for b in range(B)])
    outs = []
    for perm in (False, True):
        bt = qne.Batch(m, B)
        if perm:
            table = np.random.default_rng(1).permutation(B * 256).astype(np.uint32)
            bt.set_page_table(table)
        for t in range(L):
            nxt, lg = bt.step(prompts[:, t], np.full(B, t), want_logits=True)
        outs.append((nxt.copy(), lg.copy()))
        bt.close()
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))


def test_greedy_decode_async_matches_host_steps(tiny):
    """batch_step leaves each sequence at (greedy pick, pos + 1), so the device-resident greedy
    loop continues exactly where a host-driven loop would."""
    s, m = tiny
    B, L, steps = 4, 9, 10
    prompts = np.stack([synth.prompt_ids(L, 300 + b, 8192) for b in range(B)])
    a = qne.Batch(m, B)
    h = qne.Batch(m, B)
    for t in range(L):
        nxt_a = a.step(prompts[:, t], np.full(B, t))
        nxt_h = h.step(prompts[:, t], np.full(B, t))
    assert np.array_equal(nxt_a, nxt_h)
    tok, pos = a.tokens()
    assert np.array_equal(tok, nxt_a) and np.all(pos == L)
    dev_ids, host_ids = [], []
    cur = nxt_h.copy()
    for i in range(steps):
        a.decode_async(1)
        dev_ids.append(a.tokens()[0].copy())
        cur = h.step(cur, np.full(B, L + i))
        host_ids.append(cur.copy())
    assert np.array_equal(np.stack(dev_ids), np.stack(host_ids))
    a.close()
    h.close()


def test_context_limit_and_bad_tables(tiny):
    s, m = tiny
    bt = qne.Batch(m, 2)
    with pytest.raises(qne.QneError) as e:
        bt.step([1, 2], [0, 4096])
    assert e.value.name == "ERANGE_CTX"
    with pytest.raises(qne.QneError) as e:
        bt.set_page_table(np.full(2 * 256, 2 * 256, np.uint32))
    assert e.value.name == "EINVAL"
    bt.fill_synthetic(0, 4000, 5, 1)
    with pytest.raises(qne.QneError) as e:
        bt.decode_async(200)
    assert e.value.name == "ERANGE_CTX"
    bt.close()
    with pytest.raises(qne.QneError):
        qne.Batch(m, 33)


def _int4_matrix(kind, rows, k, rng):
    w = rng.integers(0, 1 << 32, rows * k // 8, dtype=np.uint64).astype(np.uint32)
    if kind == "q4":
        s = np.abs(rng.standard_normal(rows * k // 32) * 0.01).astype(np.float16)
        z = rng.integers(0, 1 << 32, rows * k // 256, dtype=np.uint64).astype(np.uint32)
    else:
        s = np.abs(rng.standard_normal(rows * k // 64) * 0.01).astype(np.float16)
        z = rng.uniform(0, 15, rows * k // 64).astype(np.float16)
    return w, s, z


@pytest.mark.parametrize("kind", ["q4g64", "q4"])
@pytest.mark.parametrize("batch", [1, 5, 16, 32, 33, 64])
@pytest.mark.parametrize("epilogue,rows,k", [("store", 8224, 1024), ("accumulate", 1024, 3584), ("swiglu", 2 * 3584, 1024),
                                             ("swiglu", 2 * 6144, 2048), ("accumulate", 2048, 6144), ("store", 300, 256)])
def test_int4_gemm_widens_nibbles_in_shared_memory(cuda, kind, batch, epilogue, rows, k):
    """The tensor-core GEMM on int4 weights (nibbles widened to f16 between the TMA load and the
    MMA, random zero points, partial tiles, split k) against the oracle's per-sequence GEMV."""
    rng = np.random.default_rng(batch * 11 + rows + k)
    w, s, z = _int4_matrix(kind, rows, k, rng)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal((batch, out_rows)).astype(np.float32)
    wd, sd, zd = dev(w.view(np.int32)), dev(s), dev(z.view(np.int32) if kind == "q4" else z)
    m = qne.matrix(kind, rows, k, wd, sd, zd)
    yd = dev(y0 if epilogue == "accumulate" else np.zeros((batch, out_rows), np.float32))
    qne.gemm(m, dev(x), batch, yd, epilogue, impl="tcgen05")
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    for b in range(batch):
        want = y0[b].copy() if epilogue == "accumulate" else np.zeros(out_rows, np.float32)
        oracle.gemv(kind, w, s, z, rows, k, x[b], want, rc.EPI[epilogue])
        # the GEMM multiplies the f16-rounded dequantized weights (one rounding per weight)
        assert rc.rel_err(got[b], want) < 2e-3, b


def test_int4_gemm_rejects_the_mma_sync_kernel(cuda):
    rng = np.random.default_rng(1)
    w, s, z = _int4_matrix("q4g64", 256, 256, rng)
    m = qne.matrix("q4g64", 256, 256, dev(w.view(np.int32)), dev(s), dev(z))
    x = dev(np.zeros((4, 256), np.float32))
    y = dev(np.zeros((4, 256), np.float32))
    with pytest.raises(qne.QneError) as e:
        qne.gemm(m, x, 4, y, "store", impl="mma_sync")
    assert e.value.name == "EINVAL"
    torch.cuda.synchronize()
