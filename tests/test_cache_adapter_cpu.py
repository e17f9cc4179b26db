"""Host-side checks of the Python-hook adapter (no GPU): the reference's geometry check, the
method surface the engine calls, and the bank views -> pool mapping (FTW order, gate = rows
[0, I), up = rows [I, 2I))."""
import pytest
import torch

from nvmoe_b200.cache import SlotCache, expert_gemm, pool_from_views
from nvmoe_b200.formats import random_experts


def test_geometry_check_matches_reference():
    host = random_experts("nvfp4", 2 * 8, 256, 128, seed=1)
    with pytest.raises(ValueError, match="cache_size 4 < num_experts 8"):
        SlotCache(host, 2, 8, 4, device="cpu")
    with pytest.raises(ValueError, match="host tier holds"):
        SlotCache(host, 3, 8, 8, device="cpu")


def test_surface_names():
    for name in ("ensure_experts", "copy_missing", "bank_views", "alphas_for_slots", "reset",
                 "is_cpu_layer", "slot_for_id", "id_of_slot"):
        assert hasattr(SlotCache, name)
    assert callable(expert_gemm)


def test_pool_from_views_ftw_order():
    w = random_experts("nvfp4", 4, 256, 128, seed=2)
    p = pool_from_views(w.banks(), "nvfp4", 256, 128)
    assert p.gate_up.data.data_ptr() == w.gate_up.data.data_ptr()
    assert p.down.scale.data_ptr() == w.down.scale.data_ptr()
    assert p.gate_up.glob.shape == (4,) and p.down.glob.shape == (4,)
    assert p.gate_up.rows == 256 and p.down.rows == 256 and p.n_slots == 4


def test_pool_from_views_gguf_and_bf16():
    for q in ("q2_k", "iq2_xxs", "bf16"):
        w = random_experts(q, 3, 512, 256, seed=3)
        p = pool_from_views(w.banks(), q, 512, 256)
        assert p.gate_up.data.data_ptr() == w.gate_up.data.data_ptr()
        assert p.down.data.data_ptr() == w.down.data.data_ptr()
        assert p.gate_up.data.shape == w.gate_up.data.shape
        assert p.down.data.shape == w.down.data.shape


def test_hook_flow_names():
    from nvmoe_b200.cache import decode_routed, prefill_routed
    assert callable(decode_routed) and callable(prefill_routed)
    assert hasattr(SlotCache, "materialize_layer")
