"""GPU parity of the sm_100a kernels against the CPU oracle (called through the C ABI).

Integer / index work (router ids, remap, miss lists, dequantised bytes) must be bit-exact.
FFN outputs: fp32-accumulated oracle, bf16 output; tolerance written per test
(max |y - ref| <= 1e-2 * max |ref|, i.e. rel 1e-2 of the output scale, and the mean error
well below that)."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.formats import random_experts
from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import ref_numpy as R
from oracle.native import OracleLayer

pytestmark = pytest.mark.gpu

GOLD = __import__("pathlib").Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------------ R1 router
def test_router_softmax_matches_oracle(cuda_device):
    g = np.load(GOLD / "router_golden.npz")
    lg = torch.from_numpy(g["softmax_logits"]).to(cuda_device)
    ids, w = ops.router_topk(lg, 10)
    np.testing.assert_array_equal(ids.cpu().numpy(), g["softmax_ids"])
    np.testing.assert_allclose(w.cpu().numpy(), g["softmax_w"], rtol=2e-6, atol=1e-7)


def test_router_sigmoid_bias_matches_oracle(cuda_device):
    g = np.load(GOLD / "router_golden.npz")
    lg = torch.from_numpy(g["sigmoid_logits"]).to(cuda_device)
    b = torch.from_numpy(g["sigmoid_bias"]).to(cuda_device)
    ids, w = ops.router_topk(lg, 8, mode="sigmoid_bias", bias=b, norm_topk=True,
                             routed_scaling=2.5)
    np.testing.assert_array_equal(ids.cpu().numpy(), g["sigmoid_ids"])
    np.testing.assert_allclose(w.cpu().numpy(), g["sigmoid_w"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("E,k,n", [(64, 4, 33), (512, 10, 200), (288, 8, 5), (1024, 32, 3)])
def test_router_random_shapes(cuda_device, E, k, n):
    rng = np.random.default_rng(E + k)
    lg = rng.standard_normal((n, E)).astype(np.float32)
    lg[0, :5] = 7.0  # exact ties -> lower id
    ids, w = ops.router_topk(torch.from_numpy(lg).to(cuda_device), k)
    rids, rw = R.router_topk_softmax(lg, k)
    np.testing.assert_array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    ids2, w2 = ops.router_topk(torch.from_numpy(lg).to(cuda_device), k, norm_topk=False)
    rids2, rw2 = R.router_topk_softmax(lg, k, norm_topk=False)
    np.testing.assert_array_equal(ids2.cpu().numpy(), rids2)
    np.testing.assert_allclose(w2.cpu().numpy(), rw2, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("E,k", [(513, 32), (700, 10), (1000, 8), (1024, 16), (300, 10)])
def test_router_edge_rows(cuda_device, E, k):
    """Ties inside and across the two 512-expert halves of long rows, +0/-0 ties, NaN and -inf
    logits, a short second half (E = 513); both router modes."""
    rng = np.random.default_rng(E * 7 + k)
    lg = rng.standard_normal((6, E)).astype(np.float32)
    top = [5, E - 1, min(511, E - 1), min(512, E - 1), E // 2, 3]
    lg[0, top] = 9.0                                     # six-way tie, ids across both halves
    lg[1, :] = 0.0
    lg[1, ::3] = -0.0                                    # +0 / -0 compare equal -> lower id
    lg[2, ::5] = np.nan                                  # NaN never wins
    lg[3, 1::2] = -np.inf
    lg[4, :] = np.float32(1.25)                          # every key equal
    lg[4, E - 1] = 1.5
    t = torch.from_numpy(lg).to(cuda_device)
    ids, w = ops.router_topk(t, k)
    rids, rw = R.router_topk_softmax(lg, k)
    np.testing.assert_array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    b = (rng.standard_normal(E) * 0.1).astype(np.float32)
    b[top] = 0.0
    ids2, w2 = ops.router_topk(t, k, mode="sigmoid_bias", bias=torch.from_numpy(b).to(cuda_device),
                               norm_topk=True, routed_scaling=2.5)
    rids2, rw2, _ = R.router_topk_sigmoid_bias(lg, k, b, True, 2.5)
    np.testing.assert_array_equal(ids2.cpu().numpy(), rids2)
    np.testing.assert_allclose(w2.cpu().numpy(), rw2, rtol=2e-6, atol=1e-7)


# ------------------------------------------------------------------ R2/R3/R6 remap
def _run_trace(dev, name, gold):
    E, k, S, pinned, n_tok, steps = gold[f"{name}_meta"].tolist()
    table = ops.SlotTableGPU(E, S, dev, pinned_k=pinned)
    for st in range(steps):
        ids = torch.from_numpy(gold[f"{name}_ids"][st]).to(dev)
        slots, ml = ops.remap(table, ids, is_decode=True)
        h = ml.to_host()
        assert h["status"] == 0
        np.testing.assert_array_equal(slots.cpu().numpy(), gold[f"{name}_slots"][st])
        m = int(gold[f"{name}_nmiss"][st])
        assert h["n_miss"] == m
        np.testing.assert_array_equal(h["miss_ids"], gold[f"{name}_miss_ids"][st][:m])
        np.testing.assert_array_equal(h["miss_slots"], gold[f"{name}_miss_slots"][st][:m])
        np.testing.assert_array_equal(h["evicted"], gold[f"{name}_evicted"][st][:m])


@pytest.mark.parametrize("name", ["cfg1_b1", "cfg1_b3", "cfg2_b1", "cfg2_b8"])
def test_remap_matches_golden_traces(cuda_device, name):
    _run_trace(cuda_device, name, np.load(GOLD / "remap_traces.npz"))


@pytest.mark.parametrize("E,k,S,pinned,n_tok,decode", [
    (64, 4, 16, 0, 4, True), (512, 10, 128, 4, 8, True), (512, 10, 128, 8, 12, False),
    (288, 8, 36, 2, 4, True), (512, 10, 512, 0, 64, True), (256, 8, 32, 3, 3, True),
])
def test_remap_random_vs_oracle(cuda_device, E, k, S, pinned, n_tok, decode):
    rng = np.random.default_rng(E * 7 + S)
    bias = layer_log_bias(1, E, 1.1, seed=S)[0]
    table = ops.SlotTableGPU(E, S, cuda_device, pinned_k=pinned)
    orc = OracleLayer(E, S, pinned)
    for st in range(60):
        ids_np, _ = R.router_topk_softmax(router_logits(n_tok, bias, rng), k)
        if len(np.unique(ids_np)) > S:
            continue
        # strided rows: a column slice of a wider buffer (ggml nb[1] != k*4)
        wide = torch.full((n_tok, k + 5), -7, dtype=torch.int32, device=cuda_device)
        wide[:, 2:2 + k] = torch.from_numpy(ids_np).to(cuda_device)
        view = wide[:, 2:2 + k]
        slots, ml = ops.remap(table, view, is_decode=decode, out=view)  # in place
        ref = orc.eval(ids_np.reshape(-1), is_decode=decode)
        h = ml.to_host()
        assert h["status"] == 0 and ref["status"] == 0
        np.testing.assert_array_equal(view.cpu().numpy(), ref["slots"].reshape(n_tok, k))
        assert (wide[:, :2] == -7).all() and (wide[:, 2 + k:] == -7).all()
        np.testing.assert_array_equal(h["unique_ids"], ref["unique_ids"])
        np.testing.assert_array_equal(h["unique_hit"], ref["unique_hit"])
        np.testing.assert_array_equal(h["miss_ids"], ref["miss_ids"])
        np.testing.assert_array_equal(h["miss_slots"], ref["miss_slots"])
        np.testing.assert_array_equal(h["evicted"], ref["evicted"])
        a, b, c, step = orc.tables()
        np.testing.assert_array_equal(table.slot_of_real.cpu().numpy(), a)
        np.testing.assert_array_equal(table.real_in_slot.cpu().numpy(), b)
        np.testing.assert_array_equal(table.last_used.cpu().numpy().view(np.uint32), c)
        assert int(table.step.item()) == step


def test_remap_errors_leave_tables_untouched(cuda_device):
    table = ops.SlotTableGPU(64, 8, cuda_device)
    ids = torch.tensor([[1, 2, 3, 4]], dtype=torch.int32, device=cuda_device)
    ops.remap(table, ids, True)
    snap = [t.clone() for t in (table.slot_of_real, table.real_in_slot, table.last_used, table.step)]
    bad = torch.tensor([[1, 64, 3, 4]], dtype=torch.int32, device=cuda_device)
    _, ml = ops.remap(table, bad, True)
    assert ml.to_host()["status"] == -2
    over = torch.arange(9, dtype=torch.int32, device=cuda_device).view(1, 9)
    _, ml = ops.remap(table, over, True)
    assert ml.to_host()["status"] == -3
    for a, b in zip(snap, (table.slot_of_real, table.real_in_slot, table.last_used, table.step)):
        assert torch.equal(a, b)


def test_remap_global_pool_id_base(cuda_device):
    """Python engine: one slot pool shared by all layers, id = layer*E + e
    (nvme_offload_cache.py:1431 id_base)."""
    L, E, S = 3, 16, 8
    table = ops.SlotTableGPU(L * E, S, cuda_device)
    orc = OracleLayer(L * E, S, 0)
    rng = np.random.default_rng(5)
    for st in range(40):
        layer = st % L
        ids_np = rng.choice(E, size=4, replace=False).astype(np.int32).reshape(1, 4)
        slots, ml = ops.remap(table, torch.from_numpy(ids_np).to(cuda_device), True,
                              id_base=layer * E, n_expert=E)
        ref = orc.eval((ids_np + layer * E).reshape(-1), True)
        np.testing.assert_array_equal(slots.cpu().numpy().reshape(-1), ref["slots"])


# ------------------------------------------------------------------ R8 dequant
def test_dequant_bit_exact(cuda_device):
    g = np.load(GOLD / "dequant_golden.npz")
    q2 = ops.dequant_q2_k(torch.from_numpy(g["q2k_blocks"]).to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(q2.view(np.uint32), g["q2k_values"].view(np.uint32))
    iq = ops.dequant_iq2_xxs(torch.from_numpy(g["iq2xxs_blocks"]).to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(iq.view(np.uint32), g["iq2xxs_values"].view(np.uint32))
    nv = ops.dequant_nvfp4(torch.from_numpy(g["nvfp4_codes"]).to(cuda_device),
                           torch.from_numpy(g["nvfp4_scales"]).to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(nv.view(np.uint32), g["nvfp4_values_noglobal"].view(np.uint32))


@pytest.mark.parametrize("quant", ["nvfp4", "q2_k", "iq2_xxs"])
def test_dequant_random_banks_bit_exact(cuda_device, quant):
    w = random_experts(quant, 2, 512, 256, seed=3)
    m = w.down  # [2, 512, 256 cols]
    if quant == "nvfp4":
        glob = m.glob[1:2].to(cuda_device)
        got = ops.dequant_nvfp4(m.data[1].to(cuda_device), m.scale[1].to(cuda_device), glob)
        ref = R.dequant_nvfp4(m.data[1].numpy(), m.scale[1].numpy(), m.glob[1].item())
    elif quant == "q2_k":
        got = ops.dequant_q2_k(m.data[1].to(cuda_device))
        ref = R.dequant_q2_k(m.data[1].numpy())
    else:
        from nvmoe_b200.formats import iq2xxs_grid
        got = ops.dequant_iq2_xxs(m.data[1].to(cuda_device))
        ref = R.dequant_iq2_xxs(m.data[1].numpy(), iq2xxs_grid())
    got = got.cpu().numpy().reshape(-1)
    np.testing.assert_array_equal(got.view(np.uint32), ref.reshape(-1).view(np.uint32))


# ------------------------------------------------------------------ R7/R9 FFN
def _dense(w, which, s):
    """oracle dense fp32 weights of slot s: gate [I,H], up [I,H], down [H,I]"""
    I = w.inter
    if which in ("gate", "up"):
        m = w.gate_up
        rows = slice(0, I) if which == "gate" else slice(I, 2 * I)
    else:
        m = w.down
        rows = slice(None)
    if w.quant == "nvfp4":
        return R.dequant_nvfp4(m.data[s, rows].numpy(), m.scale[s, rows].numpy(),
                               m.glob[s].item())
    if w.quant == "q2_k":
        d = m.data[s, rows].numpy()
        return R.dequant_q2_k(d).reshape(d.shape[0], -1)
    from nvmoe_b200.formats import iq2xxs_grid
    d = m.data[s, rows].numpy()
    return R.dequant_iq2_xxs(d, iq2xxs_grid()).reshape(d.shape[0], -1)


def _oracle_ffn(w, x, slots, wts, shared=None, sgate=None):
    cache = {}

    def get(which, s):
        key = (which, s)
        if key not in cache:
            cache[key] = _dense(w, which, s)
        return cache[key]

    sh = None
    if shared is not None:
        sh = (_dense(shared, "gate", 0), _dense(shared, "up", 0), _dense(shared, "down", 0))
    return R.moe_ffn(x.view(torch.int16).numpy().view(np.uint16), slots, wts,
                     lambda s: get("gate", s), lambda s: get("up", s), lambda s: get("down", s),
                     sh, None if sgate is None else sgate.view(torch.int16).numpy().view(np.uint16))


def _check_ffn(y, ref):
    y = y.float().cpu().numpy()
    scale = float(np.abs(ref).max())
    err = np.abs(y - ref)
    assert scale > 0
    assert err.max() <= 1e-2 * scale, (err.max(), scale)
    assert err.mean() <= 2e-3 * scale, (err.mean(), scale)


@pytest.mark.parametrize("n_tok,k,shared,sgate", [
    (1, 10, True, False), (2, 10, True, True), (8, 10, True, False), (13, 4, False, False),
    (64, 10, True, True), (33, 8, False, False),
])
def test_ffn_nvfp4_matches_oracle(cuda_device, n_tok, k, shared, sgate):
    H, I, S = 2048, 512, 24
    w = random_experts("nvfp4", S, H, I, seed=n_tok)
    sw = random_experts("nvfp4", 1, H, I, seed=1000 + n_tok) if shared else None
    rng = np.random.default_rng(n_tok)
    x = torch.from_numpy(rng.standard_normal((n_tok, H)).astype(np.float32)).to(torch.bfloat16)
    slots = np.stack([rng.choice(S, size=k, replace=False) for _ in range(n_tok)]).astype(np.int32)
    wts = rng.random((n_tok, k)).astype(np.float32)
    wts /= wts.sum(1, keepdims=True)
    g = (torch.from_numpy(rng.standard_normal(H).astype(np.float32) * 0.05).to(torch.bfloat16)
         if sgate else None)
    y = ops.moe_ffn(w.to(cuda_device), x.to(cuda_device), torch.from_numpy(slots).to(cuda_device),
                    torch.from_numpy(wts).to(cuda_device),
                    shared=None if sw is None else sw.to(cuda_device),
                    shared_gate=None if g is None else g.to(cuda_device))
    torch.cuda.synchronize()
    _check_ffn(y, _oracle_ffn(w, x, slots, wts, sw, g))


def test_ffn_shrunk_pool_equals_full_pool(cuda_device):
    """Reference invariant (scripts/test_mul_mat_id_shrink.cpp:71-137): the FFN over a shrunk
    slot pool with remapped ids equals the FFN over the full expert tensor with real ids.
    Each expert's tiles are computed whole by one CTA and summed in a fixed order, so the
    outputs must be identical bit for bit."""
    H, I, E, S = 2048, 512, 64, 16
    full = random_experts("nvfp4", E, H, I, seed=9)
    real = np.array([[29, 10, 5, 2, 19, 63, 50, 17]], np.int32)  # 8 routed experts, 1 token
    shrunk_gu = full.gate_up.data[real[0]]
    from nvmoe_b200.formats import ExpertWeights, QuantMatrix
    pad = lambda t: torch.cat([t, torch.zeros((S - t.shape[0], *t.shape[1:]), dtype=t.dtype)])
    shr = ExpertWeights("nvfp4", H, I,
                        QuantMatrix("nvfp4", 2 * I, H, pad(full.gate_up.data[real[0]]),
                                    pad(full.gate_up.scale[real[0]]), pad(full.gate_up.glob[real[0]])),
                        QuantMatrix("nvfp4", H, I, pad(full.down.data[real[0]]),
                                    pad(full.down.scale[real[0]]), pad(full.down.glob[real[0]])))
    del shrunk_gu
    remapped = np.arange(8, dtype=np.int32).reshape(1, 8)
    x = torch.randn((1, H), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    wts = torch.full((1, 8), 0.125)
    d = cuda_device
    y_full = ops.moe_ffn(full.to(d), x.to(d), torch.from_numpy(real).to(d), wts.to(d))
    y_shr = ops.moe_ffn(shr.to(d), x.to(d), torch.from_numpy(remapped).to(d), wts.to(d))
    assert torch.equal(y_full, y_shr)


def test_ffn_deterministic_and_strided_ids(cuda_device):
    H, I, S, n, k = 2048, 512, 32, 16, 10
    w = random_experts("nvfp4", S, H, I, seed=4).to(cuda_device)
    rng = np.random.default_rng(2)
    slots = np.stack([rng.choice(S, size=k, replace=False) for _ in range(n)]).astype(np.int32)
    wide = torch.zeros((n, k + 6), dtype=torch.int32, device=cuda_device)
    wide[:, 3:3 + k] = torch.from_numpy(slots).to(cuda_device)
    x = torch.randn((n, H), device=cuda_device).to(torch.bfloat16)
    wts = torch.rand((n, k), device=cuda_device)
    y1 = ops.moe_ffn(w, x, wide[:, 3:3 + k], wts)
    y2 = ops.moe_ffn(w, x, torch.from_numpy(slots).to(cuda_device), wts)
    assert torch.equal(y1, y2)


def test_ffn_bad_slot_reports_status(cuda_device):
    H, I, S = 2048, 512, 8
    w = random_experts("nvfp4", S, H, I, seed=1).to(cuda_device)
    st = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ids = torch.tensor([[0, 1, 99]], dtype=torch.int32, device=cuda_device)
    x = torch.randn((1, H), device=cuda_device).to(torch.bfloat16)
    ops.moe_ffn(w, x, ids, torch.ones((1, 3), device=cuda_device), status=st)
    assert int(st.item()) == -8


# ------------------------------------------------------------------ R5 refill
def test_refill_async_and_gather_byte_exact(cuda_device):
    H, I, S, HS = 2048, 512, 8, 12
    host = random_experts("nvfp4", HS, H, I, seed=21)
    host_p = type(host)(host.quant, H, I,
                        type(host.gate_up)(**{**host.gate_up.__dict__,
                                              "data": host.gate_up.data.pin_memory(),
                                              "scale": host.gate_up.scale.pin_memory(),
                                              "glob": host.gate_up.glob.pin_memory()}),
                        type(host.down)(**{**host.down.__dict__,
                                           "data": host.down.data.pin_memory(),
                                           "scale": host.down.scale.pin_memory(),
                                           "glob": host.down.glob.pin_memory()}))
    gpu = random_experts("nvfp4", S, H, I, seed=22).to(cuda_device)
    banks = ops.refill_banks(gpu, host_p)
    cs = torch.cuda.Stream()
    ev = torch.cuda.Event()
    gs, hs = [3, 4, 0], [7, 8, 11]
    ops.refill_async(banks, gs, hs, S, HS, cs, torch.cuda.current_stream(), ev)
    torch.cuda.synchronize()
    for g_, h_ in zip(gs, hs):
        assert torch.equal(gpu.gate_up.data[g_].cpu(), host.gate_up.data[h_])
        assert torch.equal(gpu.gate_up.scale[g_].cpu(), host.gate_up.scale[h_])
        assert torch.equal(gpu.down.data[g_].cpu(), host.down.data[h_])
        assert torch.equal(gpu.down.glob[g_].cpu(), host.down.glob[h_])
    # device-driven gather: miss list from the remap kernel, host slot per expert id
    table = ops.SlotTableGPU(HS, S, cuda_device)
    ids = torch.tensor([[5, 9, 2]], dtype=torch.int32, device=cuda_device)
    _, ml = ops.remap(table, ids, True)
    host_slot_of_id = torch.arange(HS, dtype=torch.int32, device=cuda_device)
    # global scale rows are 4 bytes: the gather needs 16-byte rows, so gather codes + scales
    banks16 = [b for b in banks if b.row_bytes % 16 == 0]
    ops.refill_gather(banks16, ml, host_slot_of_id, S)
    torch.cuda.synchronize()
    h = ml.to_host()
    assert h["status"] == 0
    for e, s in zip(h["miss_ids"], h["miss_slots"]):
        assert torch.equal(gpu.gate_up.data[s].cpu(), host.gate_up.data[e])
        assert torch.equal(gpu.down.scale[s].cpu(), host.down.scale[e])


def test_fp4_mma_probe_rate_is_sane(cuda_device):
    """nvmoe_probe_fp4_mma completes (bounded wait, status 0) and measures a block-scaled FP4
    MMA rate between 1 and 12 PFLOP/s (B200 nominal dense FP4: 9 PFLOP/s)."""
    tf = ops.fp4_mma_tflops(n_iter=1024, reps=2, device=cuda_device)
    assert 1000.0 < tf < 12000.0, tf
