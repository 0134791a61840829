"""Operator parity on the B200: every CUDA kernel, through the C ABI, against the CPU oracle
(and, for the reference's own self-check inputs, against the golden fixtures)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import qne
import refchecks as rc
from oracle import oracle

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "reference_checks.npz")


_SIGNED = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32, np.dtype(np.uint64): np.int64}


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype in _SIGNED:
        a = a.view(_SIGNED[a.dtype])
    return torch.from_numpy(a).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


_KEEP = []


def devmat(kind, rows, k, w, s=None, z=None):
    """Matrix descriptor over device copies that stay alive until the module ends (the descriptor
    holds raw pointers; a freed block would be handed to the next allocation)."""
    tw = dev(w)
    ts = None if s is None else dev(s)
    tz = None if z is None else dev(z)
    _KEEP.append((tw, ts, tz))
    if len(_KEEP) > 64:
        torch.cuda.synchronize()
        del _KEEP[:32]
    return qne.matrix(kind, rows, k, tw, ts, tz)


@pytest.fixture(scope="module")
def cases():
    return rc.replay()


# ------------------------------------------------------------------------------------------
# GEMV
# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("i", range(len(rc.GEMV_ORDER)))
def test_gemv_reference_checks(cuda, cases, i):
    c = cases["gemv"][i]
    out_rows = c.rows // 2 if c.epilogue == "swiglu" else c.rows
    m = devmat("q4", c.rows, c.k, c.w, c.s, c.z)
    y = dev(c.y0 if c.epilogue == "accumulate" else np.zeros(out_rows, np.float32))
    x = dev(c.x)
    qne.gemv(m, x, y, c.epilogue)
    assert rc.rel_err(host(y), GOLDEN[c.name]) < rc.TOL_GEMV


def make_matrix(kind, rows, k, rng, zp_random=False):
    if kind == "f16":
        return dict(w=rng.standard_normal(rows * k).astype(np.float16), s=None, z=None)
    w = rng.integers(0, 1 << 32, rows * k // 8, dtype=np.uint64).astype(np.uint32)
    if kind == "q4":
        s = np.abs(rng.standard_normal(rows * k // 32) * 0.01).astype(np.float16)
        z = (rng.integers(0, 1 << 32, rows * k // 256, dtype=np.uint64).astype(np.uint32) if zp_random
             else np.full(rows * k // 256, 0x88888888, np.uint32))
        return dict(w=w, s=s, z=z)
    s = np.abs(rng.standard_normal(rows * k // 64) * 0.01).astype(np.float16)
    z = (rng.uniform(0, 15, rows * k // 64).astype(np.float16) if zp_random
         else np.full(rows * k // 64, 8, np.float16))
    return dict(w=w, s=s, z=z)


def run_gemv(kind, mat, rows, k, x, epilogue, y0=None, norm=None):
    m = devmat(kind, rows, k, mat["w"], mat["s"], mat["z"])
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y = dev(y0 if y0 is not None else np.zeros(out_rows, np.float32))
    xd = dev(x)
    if norm is None:
        qne.gemv(m, xd, y, epilogue)
    else:
        nd = dev(norm)
        qne.rmsnorm_gemv(m, xd, nd, y, epilogue)
    return host(y)


def oracle_gemv(kind, mat, rows, k, x, epilogue, y0=None):
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y = y0.copy() if y0 is not None else np.zeros(out_rows, np.float32)
    return oracle.gemv(kind, mat["w"], mat["s"], mat["z"], rows, k, x, y, rc.EPI[epilogue])


# benchmark config 5 shapes (K x N): 2048x6144, 6144x2048, 2048x4096, 1024x248320.
SHAPES = [(6144, 2048), (2048, 6144), (4096, 2048), (248320, 1024)]


@pytest.mark.parametrize("kind", ["f16", "q4g64", "q4"])
@pytest.mark.parametrize("rows,k", SHAPES)
def test_gemv_microbench_shapes(cuda, kind, rows, k):
    rng = np.random.default_rng(4)
    mat = make_matrix(kind, rows, k, rng)
    x = rng.standard_normal(k).astype(np.float32)
    got = run_gemv(kind, mat, rows, k, x, "store")
    want = oracle_gemv(kind, mat, rows, k, x, "store")
    assert rc.rel_err(got, want) < 1e-4


@pytest.mark.parametrize("kind", ["f16", "q4g64", "q4"])
@pytest.mark.parametrize("epilogue", ["store", "accumulate", "swiglu"])
@pytest.mark.parametrize("rows,k", [(2 * 3584, 1024), (74, 1024), (2, 2048), (1022, 3584), (3000, 256)])
def test_gemv_epilogues_and_tails(cuda, kind, epilogue, rows, k):
    rng = np.random.default_rng(rows + k)
    mat = make_matrix(kind, rows, k, rng, zp_random=True)
    x = rng.standard_normal(k).astype(np.float32)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal(out_rows).astype(np.float32) if epilogue == "accumulate" else None
    got = run_gemv(kind, mat, rows, k, x, epilogue, y0)
    want = oracle_gemv(kind, mat, rows, k, x, epilogue, y0)
    assert rc.rel_err(got, want) < 1e-4


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("epilogue", ["store", "accumulate", "swiglu"])
@pytest.mark.parametrize("rows,k", [(12288, 2048), (2048, 6144), (2 * 3584, 1024), (300, 6144), (2, 256), (16, 256)])
def test_gemv_variants_match_the_oracle(cuda, variant, epilogue, rows, k):
    """The selectable f16 kernels (1: the older register kernel, 2: the bulk-copy ring with one
    producer warp per CTA) compute what the default kernel computes, tails and pieces included."""
    if epilogue == "swiglu" and 4 * k > 16384 and variant == 2:
        pytest.skip("a SwiGLU row pair of this width does not fit a ring slot")
    rng = np.random.default_rng(rows * 7 + k)
    mat = make_matrix("f16", rows, k, rng)
    x = rng.standard_normal(k).astype(np.float32)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal(out_rows).astype(np.float32) if epilogue == "accumulate" else None
    m = devmat("f16", rows, k, mat["w"])
    y = dev(y0 if y0 is not None else np.zeros(out_rows, np.float32))
    qne.gemv_ex(m, dev(x), y, epilogue, variant)
    want = oracle_gemv("f16", mat, rows, k, x, epilogue, y0)
    assert rc.rel_err(host(y), want) < 1e-4


@pytest.mark.parametrize("variant", [3, 4])
@pytest.mark.parametrize("kind", ["q4g64", "q4"])
@pytest.mark.parametrize("epilogue", ["store", "accumulate", "swiglu"])
@pytest.mark.parametrize("rows,k", [(12288, 2048), (2048, 6144), (2 * 3584, 1024), (1024, 3584), (8224, 2048),
                                    (300, 6144), (74, 1024), (2, 256), (16, 256)])
def test_gemv_int4_variants(cuda, variant, kind, epilogue, rows, k):
    """Variant 3 (tensor-core int4: per-block MMA columns, slices held in registers, the default)
    and variant 4 (the CUDA-core register pipeline) against the oracle: random zero points,
    partial last tiles and every k-slice split the launcher picks."""
    if variant == 4 and epilogue == "swiglu" and k > 4096:
        pytest.skip("the register pipeline holds a SwiGLU row pair of at most 4096 values")
    rng = np.random.default_rng(rows * 3 + k)
    mat = make_matrix(kind, rows, k, rng, zp_random=True)
    x = rng.standard_normal(k).astype(np.float32)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal(out_rows).astype(np.float32) if epilogue == "accumulate" else None
    m = devmat(kind, rows, k, mat["w"], mat["s"], mat["z"])
    y = dev(y0 if y0 is not None else np.zeros(out_rows, np.float32))
    qne.gemv_ex(m, dev(x), y, epilogue, variant)
    want = oracle_gemv(kind, mat, rows, k, x, epilogue, y0)
    assert rc.rel_err(host(y), want) < 1e-4


def test_gemv_ring_variant_rejects_wide_rows(cuda):
    m = devmat("f16", 64, 8192, np.zeros(64 * 8192, np.float16))
    with pytest.raises(qne.QneError) as e:
        qne.gemv_ex(m, dev(np.zeros(8192, np.float32)), dev(np.zeros(64, np.float32)), "store", 2)
    assert e.value.name == "EINVAL"


@pytest.mark.parametrize("kind", ["f16", "q4g64", "q4"])
def test_rmsnorm_prologue(cuda, kind):
    rng = np.random.default_rng(11)
    rows, k = 5120, 2048
    mat = make_matrix(kind, rows, k, rng)
    h = (rng.standard_normal(k) * 3).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    got = run_gemv(kind, mat, rows, k, h, "store", norm=g)
    want = oracle_gemv(kind, mat, rows, k, oracle.rmsnorm(h, g), "store")
    assert rc.rel_err(got, want) < 1e-4


def test_gemv_rejects_bad_shapes(cuda):
    with pytest.raises(qne.QneError) as e:
        m = devmat("f16", 100, 100, np.zeros(100 * 100, np.float16))
        qne.gemv(m, dev(np.zeros(100, np.float32)), dev(np.zeros(100, np.float32)))
    assert e.value.name == "EINVAL"


# ------------------------------------------------------------------------------------------
# int4 unpack: bit-exact
# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("kind", ["q4", "q4g64", "f16"])
def test_dequant_bit_exact(cuda, kind):
    rng = np.random.default_rng(21)
    rows, k = 300, 1024
    mat = make_matrix(kind, rows, k, rng, zp_random=True)
    m = devmat(kind, rows, k, mat["w"], mat["s"], mat["z"])
    out = torch.empty((rows - 5, k), dtype=torch.float32, device="cuda")
    qne.dequant_rows(m, 5, rows - 5, out)
    want = oracle.dequant_rows(kind, mat["w"], mat["s"], mat["z"], rows, k, 5, rows - 5)
    got = host(out)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_embed_reference_check(cuda, cases):
    e = cases["embed"]
    m = devmat("q4", 300, 1024, e["w"], e["s"], e["z"])
    tok = dev(np.array([7, 41, 0, 0], np.uint32))
    h = torch.empty(1024, dtype=torch.float32, device="cuda")
    qne.embed(m, tok, h)
    assert np.array_equal(host(h), GOLDEN["embed"])


# ------------------------------------------------------------------------------------------
# Greedy pick: bit-exact token selection
# ------------------------------------------------------------------------------------------
def gpu_argmax(logits, tok0=(0, 41)):
    n = logits.size
    nbytes = qne.argmax_scratch_bytes(n)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    tok = dev(np.array([tok0[0], tok0[1], 0, 0], np.uint32))
    qne.argmax(dev(logits), n, tok, scratch, nbytes)
    return host(tok)


def test_argmax_known_answer(cuda, cases):
    tok = gpu_argmax(cases["embed"]["logits"], (7, 41))
    assert list(tok[:2]) == list(GOLDEN["argmax_tok"]) == [123457, 42]


@pytest.mark.parametrize("n", [1, 31, 1024, 1025, 248320, 1 << 20])
def test_argmax_ties_nan_and_sizes(cuda, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    m = x.max() + 1
    hits = sorted(set(rng.integers(0, n, 5).tolist()))
    x[hits] = m
    if n > 10:
        x[rng.integers(0, n, 3)] = np.nan
        x[hits[0]] = m
    assert gpu_argmax(x)[0] == oracle.argmax(x) == hits[0]
    for _ in range(3):  # the completion counter resets itself
        assert gpu_argmax(x)[0] == hits[0]


def test_argmax_all_negative_infinity_picks_zero(cuda):
    x = np.full(5000, -np.inf, np.float32)
    assert gpu_argmax(x)[0] == oracle.argmax(x) == 0


# ------------------------------------------------------------------------------------------
# Gated DeltaNet
# ------------------------------------------------------------------------------------------
def ring_from_reference(conv_state, count):
    """Reference window conv_state[c*3 + i] (i = 0 oldest) -> ring [4][6144] for counter `count`."""
    ring = np.zeros((4, 6144), np.float32)
    for i in range(3):
        ring[(count - 4 + i) % 4] = conv_state[i::3]
    return ring


def test_gdn_reference_check(cuda, cases):
    g = cases["gdn"]
    count = 4
    ring = dev(ring_from_reference(g["conv0"], count))
    state = dev(g["state0"])
    out = torch.empty(2048, dtype=torch.float32, device="cuda")
    ctr = dev(np.array([count], np.uint32))
    qne.gdn_step(dev(g["proj"]), ring, dev(g["conv_w"]), state, dev(g["params"]), ctr, out, 1)
    assert rc.rel_err(host(out), GOLDEN["gdn_output"]) < rc.TOL_GDN_OUT
    st = host(state)
    assert rc.rel_err(st[::61], GOLDEN["gdn_state_sample"]) < rc.TOL_GDN_STATE
    conv = g["conv0"].copy()
    st_o = g["state0"].copy()
    want = oracle.gdn_step(g["proj"], conv, g["conv_w"], st_o, g["params"])
    assert rc.rel_err(host(out), want) < 1e-4
    assert rc.rel_err(st, st_o) < 1e-5
    assert np.array_equal(host(ring)[(count - 1) % 4], g["proj"][:6144])


def test_gdn_multi_step_batched(cuda):
    rng = np.random.default_rng(3)
    B, steps = 3, 7
    conv_w = rng.uniform(-0.5, 0.5, 6144 * 4).astype(np.float32)
    params = np.concatenate([rng.uniform(-1, 1, 16), -rng.uniform(0.1, 1, 16), rng.uniform(0.5, 1.5, 128)]).astype(np.float32)
    ref_conv = [np.zeros(6144 * 3, np.float32) for _ in range(B)]
    ref_state = [(rng.standard_normal(16 * 16384) * 0.1).astype(np.float32) for _ in range(B)]
    ring = dev(np.zeros((B, 4, 6144), np.float32))
    state = dev(np.stack(ref_state))
    out = torch.empty((B, 2048), dtype=torch.float32, device="cuda")
    for n in range(1, steps + 1):
        proj = rng.standard_normal((B, 8224)).astype(np.float32)
        ctr = dev(np.full(B, n, np.uint32))
        qne.gdn_step(dev(proj), ring, dev(conv_w), state, dev(params), ctr, out, B)
        got = host(out)
        for b in range(B):
            want = oracle.gdn_step(proj[b], ref_conv[b], conv_w, ref_state[b], params)
            assert rc.rel_err(got[b], want) < 1e-4, (n, b)
    st = host(state)
    for b in range(B):
        assert rc.rel_err(st[b], ref_state[b]) < 1e-5


# ------------------------------------------------------------------------------------------
# Attention over the paged f16 cache
# ------------------------------------------------------------------------------------------
PAGE = 16
PAGE_ELEMS = 2 * 2 * PAGE * 256


def pages_from_contiguous(kc, vc, length, table, pool_pages):
    """Contiguous [2][4096][256] caches -> f16 page pool (bit pattern of f16-rounded values)."""
    pool = np.zeros((pool_pages, 2, 2, PAGE, 256), np.float16)
    for l in range(length):
        p = table[l // PAGE]
        pool[p, 0, :, l % PAGE] = kc[:, l].astype(np.float16)
        pool[p, 1, :, l % PAGE] = vc[:, l].astype(np.float16)
    return pool


def attention_case(rng, pos, batch_table_seed):
    proj = rng.standard_normal(5120).astype(np.float32)
    kc = rng.standard_normal((2, 4096, 256)).astype(np.float32)
    vc = rng.standard_normal((2, 4096, 256)).astype(np.float32)
    return proj, kc, vc


@pytest.mark.parametrize("impl", ["tensor_core", "cuda_core"])
@pytest.mark.parametrize("pos", [0, 1, 15, 16, 17, 63, 64, 65, 127, 128, 200, 1000, 2047, 4095])
def test_attention_positions_permuted_pages(cuda, pos, impl):
    rng = np.random.default_rng(pos)
    pool_pages = 300
    table = rng.permutation(pool_pages)[:256].astype(np.uint32)
    proj = rng.standard_normal(5120).astype(np.float32)
    kc = rng.standard_normal((2, 4096, 256)).astype(np.float32)
    vc = rng.standard_normal((2, 4096, 256)).astype(np.float32)
    norms = rng.uniform(0.5, 1.5, 512).astype(np.float32)
    kc16 = kc.astype(np.float16).astype(np.float32)
    vc16 = vc.astype(np.float16).astype(np.float32)
    pool = dev(pages_from_contiguous(kc16, vc16, pos, table, pool_pages).view(np.uint16))
    out = torch.empty(2048, dtype=torch.float32, device="cuda")
    nbytes = qne.attention_scratch_bytes(1)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    qne.attention_step(dev(proj), dev(norms), 1e7, pool, pool_pages, dev(table), dev(np.array([pos], np.uint32)),
                       out, 1, scratch, nbytes, impl=impl)
    rope = oracle.rope_table(1e7)
    want = oracle.attention_step(proj, kc16, vc16, pos, norms, rope, kv_f16=True)
    assert rc.rel_err(host(out), want) < 1e-4
    # the appended slot holds the f16 key/value the oracle wrote (value bit-exact, key within 1 ulp)
    pg = host(pool).view(np.float16).reshape(pool_pages, 2, 2, PAGE, 256)
    p, slot = table[pos // PAGE], pos % PAGE
    assert np.array_equal(pg[p, 1, :, slot].view(np.uint16), vc16[:, pos].astype(np.float16).view(np.uint16))
    kd = np.abs(pg[p, 0, :, slot].view(np.uint16).astype(np.int32) - kc16[:, pos].astype(np.float16).view(np.uint16).astype(np.int32))
    assert kd.max() <= 1


def test_attention_reference_check(cuda, cases):
    a = cases["attention"]
    pos, pool_pages = a["pos"], 256
    table = np.arange(256, dtype=np.uint32)
    kc = a["kc"].reshape(2, 4096, 256)
    vc = a["vc"].reshape(2, 4096, 256)
    pool = dev(pages_from_contiguous(kc, vc, pos, table, pool_pages).view(np.uint16))
    out = torch.empty(2048, dtype=torch.float32, device="cuda")
    nbytes = qne.attention_scratch_bytes(1)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    qne.attention_step(dev(a["proj"]), dev(a["norms"]), 1e7, pool, pool_pages, dev(table),
                       dev(np.array([pos], np.uint32)), out, 1, scratch, nbytes)
    # f16 cache against the reference's f32 formulas
    assert rc.rel_err(host(out), GOLDEN["attention"]) < 2e-3


@pytest.mark.parametrize("impl", ["tensor_core", "cuda_core"])
def test_attention_batched_ragged(cuda, impl):
    rng = np.random.default_rng(9)
    B, pool_pages = 5, 5 * 256
    pos = np.array([0, 16, 333, 2500, 4095], np.uint32)
    tables = rng.permutation(pool_pages).astype(np.uint32).reshape(B, 256)
    proj = rng.standard_normal((B, 5120)).astype(np.float32)
    norms = rng.uniform(0.5, 1.5, 512).astype(np.float32)
    pool = np.zeros((pool_pages, 2, 2, PAGE, 256), np.float16)
    kcs, vcs = [], []
    for b in range(B):
        kc = rng.standard_normal((2, 4096, 256)).astype(np.float16).astype(np.float32)
        vc = rng.standard_normal((2, 4096, 256)).astype(np.float16).astype(np.float32)
        kcs.append(kc)
        vcs.append(vc)
        for l in range(pos[b]):
            p = tables[b, l // PAGE]
            pool[p, 0, :, l % PAGE] = kc[:, l]
            pool[p, 1, :, l % PAGE] = vc[:, l]
    dpool = dev(pool.view(np.uint16))
    out = torch.empty((B, 2048), dtype=torch.float32, device="cuda")
    nbytes = qne.attention_scratch_bytes(B)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    rope = oracle.rope_table(1e7)
    for rep in range(2):  # the completion counters reset themselves
        qne.attention_step(dev(proj), dev(norms), 1e7, dpool, pool_pages, dev(tables), dev(pos), out, B, scratch,
                           nbytes, impl=impl)
        got = host(out)
        for b in range(B):
            want = oracle.attention_step(proj[b], kcs[b].copy(), vcs[b].copy(), int(pos[b]), norms, rope, True)
            assert rc.rel_err(got[b], want) < 1e-4, (rep, b)


def test_kv_gather_bit_exact(cuda):
    rng = np.random.default_rng(2)
    pool_pages, length = 64, 777
    table = rng.permutation(pool_pages)[:256 if pool_pages >= 256 else pool_pages].astype(np.uint32)
    table = np.concatenate([table, np.zeros(256 - table.size, np.uint32)])
    bits = rng.integers(0, 1 << 16, pool_pages * PAGE_ELEMS, dtype=np.uint64).astype(np.uint16)
    ok = torch.empty((2, length, 256), dtype=torch.int16, device="cuda")
    ov = torch.empty((2, length, 256), dtype=torch.int16, device="cuda")
    qne.kv_gather(dev(bits), dev(table), length, ok, ov)
    pg = bits.reshape(pool_pages, 2, 2, PAGE, 256)
    l = np.arange(length)
    want_k = pg[table[l // PAGE], 0, :, l % PAGE].transpose(1, 0, 2)
    want_v = pg[table[l // PAGE], 1, :, l % PAGE].transpose(1, 0, 2)
    assert np.array_equal(host(ok).view(np.uint16), want_k)
    assert np.array_equal(host(ov).view(np.uint16), want_v)


def test_bandwidth_probe_xor(cuda):
    rng = np.random.default_rng(0)
    data = rng.integers(0, 1 << 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    sink = dev(np.zeros(1, np.uint32))
    qne.bandwidth_probe(dev(data), data.nbytes, sink)
    want = np.bitwise_xor.reduce(data)
    assert int(host(sink).view(np.uint32)[0]) == int(want)
