"""The Python-hook adapter (nvmoe_b200.cache.SlotCache + expert_gemm) driven the way the
engine's decode patch drives the reference cache (nvme_offload_cache.py:2142-2184):
ensure_experts -> copy_missing -> _expert_gemm, with global slots shared by the layers.

Slot ids, miss lists and evictions are compared bit-exactly with the C oracle of eval_cb run
on global ids (layer * E + e); the outputs with the fp32 oracle FFN on the experts the slots
hold, within the FFN tolerance."""
import numpy as np
import pytest
import torch

from nvmoe_b200.cache import SlotCache, expert_gemm
from nvmoe_b200.engine import _pin
from nvmoe_b200.formats import random_experts
from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import ref_numpy as R
from oracle.native import OracleLayer

pytestmark = pytest.mark.gpu

L, E, K, H, I, S = 2, 64, 4, 2048, 512, 80


def _dense(w, which, g):
    m = w.gate_up if which != "down" else w.down
    rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
    return R.dequant_nvfp4(m.data[g, rows].numpy(), m.scale[g, rows].numpy(), m.glob[g].item())


@pytest.mark.parametrize("n_tok", [1, 3])
def test_slot_cache_decode_flow_matches_oracle(cuda_device, n_tok):
    host = _pin(random_experts("nvfp4", L * E, H, I, seed=21))
    cache = SlotCache(host, L, E, S, device=cuda_device)
    orc = OracleLayer(L * E, S)              # global ids, global slots, no pinned slots
    bias = layer_log_bias(L, E, 1.1, seed=4)
    rng = np.random.default_rng(n_tok)
    dense = {}

    def hd(which, g):
        if (which, g) not in dense:
            dense[(which, g)] = _dense(host, which, g)
        return dense[(which, g)]

    for step in range(8):
        for l in range(L):
            lg = router_logits(n_tok, bias[l], rng)
            rids, rw = R.router_topk_softmax(lg, K)
            ids = torch.from_numpy(rids.astype(np.int32)).to(cuda_device)
            w = torch.from_numpy(rw).to(cuda_device)
            x = torch.from_numpy(rng.standard_normal((n_tok, H)).astype(np.float32)).to(
                torch.bfloat16)
            cache.ensure_experts(l, ids)                       # in place: ids -> slots
            cache.copy_missing()
            y = expert_gemm(cache, x.to(cuda_device), w, ids, views=cache.bank_views(), n=None,
                            alphas=cache.alphas_for_slots(l), is_prefill=False)
            torch.cuda.synchronize()
            ref = orc.eval((rids + l * E).reshape(-1), is_decode=True)
            assert ref["status"] == 0
            cache.check()
            np.testing.assert_array_equal(ids.cpu().numpy().reshape(-1), ref["slots"])
            h = cache.misses.to_host()
            np.testing.assert_array_equal(h["miss_ids"] + l * E, ref["miss_ids"])
            np.testing.assert_array_equal(h["miss_slots"], ref["miss_slots"])
            np.testing.assert_array_equal(h["evicted"], ref["evicted"])
            sor, ris, _, _ = orc.tables()
            np.testing.assert_array_equal(cache.slot_for_id.cpu().numpy().reshape(-1), sor)
            np.testing.assert_array_equal(cache.id_of_slot.cpu().numpy(), ris)
            # every slot in use holds its expert's bytes, copied from the host tier
            yr = R.moe_ffn(x.view(torch.int16).numpy().view(np.uint16), ref["slots"].reshape(n_tok, K),
                           rw, lambda s: hd("gate", int(ris[s])), lambda s: hd("up", int(ris[s])),
                           lambda s: hd("down", int(ris[s])))
            yv = y.float().cpu().numpy()
            assert np.abs(yv - yr).max() <= 1e-2 * float(np.abs(yr).max())


def test_slot_cache_bank_views_are_the_pool(cuda_device):
    host = _pin(random_experts("nvfp4", L * E, H, I, seed=22))
    cache = SlotCache(host, L, E, S, device=cuda_device)
    v = cache.bank_views()
    assert len(v) == 6 and all(t.shape[0] == S for t in v)
    assert all(t.shape[0] == 16 for t in cache.bank_views(16))
    ids = torch.tensor([[3, 9, 1, 0]], dtype=torch.int32, device=cuda_device)
    cache.ensure_experts(1, ids)
    cache.copy_missing()
    torch.cuda.synchronize()
    for j, e in enumerate([3, 9, 1, 0]):
        s = int(ids[0, j])
        assert int(cache.slot_for_id[1, e]) == s and int(cache.id_of_slot[s]) == E + e
        assert torch.equal(v[0][s].cpu(), host.gate_up.data[E + e])   # codes byte-exact
        assert torch.equal(v[4][s].cpu(), host.down.scale[E + e])     # scales byte-exact
    cache.reset()
    assert int((cache.slot_for_id >= 0).sum()) == 0


def test_slot_cache_prefill_flow_matches_oracle(cuda_device):
    """prefill_routed as the narrowed-prefill patch runs it (nvme_offload_cache.py:1957-2013):
    the prompt's routed union ensured in one call, one slot_for_id gather, the grouped GEMM with
    is_prefill=True; after decode steps have filled part of the pool."""
    from nvmoe_b200.cache import decode_routed, prefill_routed
    from tests.helpers import DenseExperts, bf16_bits, within
    host = _pin(random_experts("nvfp4", L * E, H, I, seed=23))
    cache = SlotCache(host, L, E, S, device=cuda_device)
    orc = OracleLayer(L * E, S)
    bias = layer_log_bias(L, E, 1.1, seed=5)
    rng = np.random.default_rng(7)
    dense = DenseExperts(host)
    for step in range(3):  # decode steps first
        for l in range(L):
            rids, rw = R.router_topk_softmax(router_logits(2, bias[l], rng), K)
            ids = torch.from_numpy(rids.astype(np.int32)).to(cuda_device)
            x = torch.randn((2, H), device=cuda_device).to(torch.bfloat16)
            decode_routed(cache, l, x, torch.from_numpy(rw).to(cuda_device), ids)
            orc.eval((rids + l * E).reshape(-1), is_decode=True)
    T = 300
    for l in range(L):
        rids, rw = R.router_topk_softmax(router_logits(T, bias[l], rng), K)
        ids = torch.from_numpy(rids.astype(np.int32)).to(cuda_device)
        x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16)
        y = prefill_routed(cache, l, x.to(cuda_device), torch.from_numpy(rw).to(cuda_device), ids)
        torch.cuda.synchronize()
        cache.check()
        union = np.unique(rids).astype(np.int32)  # torch.unique: ascending
        ref = orc.eval(union + l * E, is_decode=True)
        assert ref["status"] == 0
        sor, ris, _, _ = orc.tables()
        np.testing.assert_array_equal(cache.slot_for_id.cpu().numpy().reshape(-1), sor)
        np.testing.assert_array_equal(ids.cpu().numpy(), rids)  # topk_ids left as they were
        yr = R.moe_ffn(bf16_bits(x), rids + l * E, rw, *dense.callables())
        assert within(y, yr) <= 1e-2


def test_materialize_layer_places_experts_at_identity_slots(cuda_device):
    """materialize_layer (nvme_offload_cache.py:1626-1682) then the non-narrowed GEMM over
    bank_views(num_experts) with the raw expert ids."""
    from tests.helpers import DenseExperts, bf16_bits, within
    host = _pin(random_experts("nvfp4", L * E, H, I, seed=24))
    cache = SlotCache(host, L, E, S, device=cuda_device)
    ids0 = torch.tensor([[3, 60, 7, 1]], dtype=torch.int32, device=cuda_device)
    cache.ensure_experts(0, ids0)
    cache.copy_missing()
    cache.materialize_layer(1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.slot_for_id[1].cpu().numpy(), np.arange(E))
    np.testing.assert_array_equal(cache.id_of_slot[:E].cpu().numpy(), E + np.arange(E))
    assert int((cache.slot_for_id[0] >= 0).sum()) == 0  # layer 0's experts were in slots < E
    rng = np.random.default_rng(8)
    rids, rw = R.router_topk_softmax(rng.standard_normal((64, E)).astype(np.float32), K)
    x = torch.from_numpy(rng.standard_normal((64, H)).astype(np.float32)).to(torch.bfloat16)
    y = expert_gemm(cache, x.to(cuda_device), torch.from_numpy(rw).to(cuda_device),
                    torch.from_numpy(rids.astype(np.int32)).to(cuda_device),
                    views=cache.bank_views(E), n=None, alphas=None, is_prefill=True)
    yr = R.moe_ffn(bf16_bits(x), rids + E, rw, *DenseExperts(host).callables())
    assert within(y, yr) <= 1e-2


def test_slot_cache_q2k_views(cuda_device):
    """A Q2_K pool through the hook: bank_views() gives (gate_up, down) super-block rows and
    expert_gemm runs the Q2_K decode kernel on them."""
    from nvmoe_b200.cache import decode_routed
    from tests.helpers import bf16_bits, within
    host = _pin(random_experts("q2_k", L * E, H, I, seed=25))
    cache = SlotCache(host, L, E, S, device=cuda_device)
    assert len(cache.bank_views()) == 2
    rng = np.random.default_rng(9)
    rids, rw = R.router_topk_softmax(rng.standard_normal((3, E)).astype(np.float32), K)
    ids = torch.from_numpy(rids.astype(np.int32)).to(cuda_device)
    x = torch.from_numpy(rng.standard_normal((3, H)).astype(np.float32)).to(torch.bfloat16)
    y = decode_routed(cache, 1, x.to(cuda_device), torch.from_numpy(rw).to(cuda_device), ids)
    torch.cuda.synchronize()

    def dq(which, g):
        m = host.gate_up if which != "down" else host.down
        rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
        b = m.data[g, rows].numpy()
        return R.dequant_q2_k(b).reshape(b.shape[0], -1)
    yr = R.moe_ffn(bf16_bits(x), rids + E, rw, lambda g: dq("gate", g), lambda g: dq("up", g),
                   lambda g: dq("down", g))
    assert within(y, yr) <= 1e-2
