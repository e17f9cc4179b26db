"""Generates the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py [--reference /root/reference]

Run in a container that has the reference tree; the fixtures travel with the repository so the
GPU tests never read the reference at run time.

  slru_traces.json  — op sequences replayed through the reference's own Python SegmentedHostLru
                      (nvme-moe-bench/nvme_offload_cache.py:333-409), imported with stub
                      freetoken / flashlib modules (those packages are not installed).
  dequant_golden.npz — random Q2_K / IQ2_XXS / NVFP4 blocks and gguf-py 0.19.0's dequantised
                      values (ggml's reference dequantizers); NVFP4 goes through the FTW ->
                      block_nvfp4 packing of scripts/convert_ftw_to_gguf.py:46-70.
  remap_traces.npz  — seeded routing traces and the CPU oracle's slot maps / miss lists
                      (oracle/remap_lru.c, a restatement of moe_cache_probe.cpp:eval_cb).
  router_golden.npz — seeded logits and the oracle's top-k ids / weights.
  glm_router_golden.npz — seeded logits and selection biases routed by the reference's own GLM
                      router (nvme_offload_cache.py:2980-3089), imported with stub modules.
"""
from __future__ import annotations

import argparse
import json
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def _stub_reference_imports() -> None:
    """Minimal stand-ins so nvme_offload_cache.py imports (only SegmentedHostLru is used)."""
    def mod(name, **attrs):
        m = types.ModuleType(name)
        for k, v in attrs.items():
            setattr(m, k, v)
        sys.modules[name] = m
        return m

    class _Base:  # OffloadMoeCache stand-in
        pass

    import logging
    mod("flashlib")
    mod("flashlib.kernels")
    mod("flashlib.kernels.slot_cache", lru_ensure=None)
    mod("freetoken")
    mod("freetoken.core", get_global_ctx=None)
    mod("freetoken.kernel")
    mod("freetoken.kernel.fast_index_copy", fast_index_copy_multi_jit=None)
    mod("freetoken.kernel.pinned", device_ptr=None)
    mod("freetoken.moe")
    mod("freetoken.moe.offload_cache", _BANK_SCHEMAS={}, MARLIN_MAX_CACHE_SIZE=0, N_STATS=1,
        OffloadMoeCache=_Base)
    mod("freetoken.moe.offload_kernels", ensure_experts=None, materialize_layer=None)
    mod("freetoken.utils", init_logger=lambda *a, **k: logging.getLogger("ref"))


def slru_traces(ref: Path, n_traces: int = 16, n_ops: int = 300) -> list:
    _stub_reference_imports()
    sys.path.insert(0, str(ref / "nvme-moe-bench"))
    import nvme_offload_cache as noc  # the reference module

    rng = np.random.default_rng(1234)
    traces = []
    for t in range(n_traces):
        ratio = float(rng.choice([0.8, 0.5, 0.25, 1.0]))
        cap = int(rng.integers(1, 40))
        n_keys = int(rng.integers(4, 64))
        lru = noc.SegmentedHostLru(protected_ratio=ratio)
        ops = []
        hint_done = False
        present: set[int] = set()
        for _ in range(n_ops):
            r = rng.random()
            if not hint_done and r < 0.05:
                lru.set_capacity_hint(cap)
                hint_done = True
                ops.append(["hint", cap, None])
                continue
            if r < 0.35:
                absent = [k for k in range(n_keys) if k not in present]
                if not absent:
                    continue
                k = int(rng.choice(absent))
                lru.insert_new(k)
                present.add(k)
                ops.append(["insert_new", k, None])
            elif r < 0.70:
                k = int(rng.integers(0, n_keys))
                lru.touch(k)
                ops.append(["touch", k, None])
            elif r < 0.82:
                if not present:
                    continue
                k, _ = lru.pop_lru()
                present.discard(k)
                ops.append(["pop_lru", None, int(k)])
            elif r < 0.92:
                if not present:
                    continue
                prot = sorted(int(x) for x in rng.choice(
                    n_keys, size=min(n_keys, int(rng.integers(0, 6))), replace=False))
                k, _ = lru.pop_lru(protect=set(prot))
                present.discard(k)
                ops.append(["pop_excluding", prot, int(k)])
            elif r < 0.97:
                k = int(rng.integers(0, n_keys))
                lru.discard(k)
                present.discard(k)
                ops.append(["discard", k, None])
            else:
                k = int(rng.integers(0, n_keys))
                ops.append(["contains", k, bool(k in lru)])
            ops.append(["size", None, len(lru)])
        traces.append({"ratio": ratio, "n_keys": n_keys, "ops": ops})
    return traces


def dequant_golden() -> dict:
    from gguf.quants import IQ2_XXS, NVFP4, Q2_K

    from nvmoe_b200.formats import ftw_to_gguf_nvfp4

    rng = np.random.default_rng(7)
    out = {}
    # Q2_K: random payload, fp16 d/dmin with a spread of magnitudes
    nb = 16
    q2 = rng.integers(0, 256, size=(nb, 84), dtype=np.uint8)
    q2[:, 80:82] = np.abs(rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    q2[:, 82:84] = np.abs(rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    out["q2k_blocks"] = q2
    out["q2k_values"] = Q2_K.dequantize_blocks(q2.copy()).reshape(-1).astype(np.float32)
    # IQ2_XXS
    iq = rng.integers(0, 256, size=(nb, 66), dtype=np.uint8)
    iq[:, 0:2] = np.abs(rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    IQ2_XXS.init_grid()
    out["iq2xxs_blocks"] = iq
    out["iq2xxs_values"] = IQ2_XXS.dequantize_blocks(iq.copy()).reshape(-1).astype(np.float32)
    out["iq2xxs_grid"] = np.asarray(IQ2_XXS.grid, np.float32).reshape(256, 8).astype(np.uint8)
    out["ksigns"] = np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()
    # NVFP4: FTW rows, scales 2^U(-8,-2) as e4m3 (incl. subnormals) + a few edge scales
    import torch
    rows, cols = 8, 256
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    sc = torch.exp2(torch.from_numpy(rng.uniform(-8, -2, size=(rows, cols // 16)).astype(np.float32)))
    scales = sc.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    scales[0, :4] = [0x00, 0x01, 0x07, 0x7E]  # zero, smallest subnormal, largest subnormal, 448
    out["nvfp4_codes"] = codes
    out["nvfp4_scales"] = scales
    blocks = ftw_to_gguf_nvfp4(codes, scales)
    out["nvfp4_values_noglobal"] = NVFP4.dequantize_blocks(
        blocks.reshape(-1, 36).copy()).reshape(rows, cols).astype(np.float32)
    return out


def remap_traces() -> dict:
    from oracle.native import OracleLayer
    from nvmoe_b200.synth import layer_log_bias, router_logits
    from oracle.ref_numpy import router_topk_softmax

    out = {}
    cases = [
        # name, E, k, S, pinned, n_tok, steps, skew
        ("cfg1_b1", 64, 4, 16, 0, 1, 200, 1.1),
        ("cfg1_b3", 64, 4, 16, 0, 3, 120, 1.1),
        ("cfg2_b8", 512, 10, 128, 4, 8, 40, 1.1),
        ("cfg2_b1", 512, 10, 128, 0, 1, 60, 1.1),
    ]
    for name, E, k, S, pinned, n_tok, steps, skew in cases:
        rng = np.random.default_rng(0)
        bias = layer_log_bias(1, E, skew, seed=0)[0]
        lay = OracleLayer(E, S, pinned)
        ids_all, slots_all, nmiss, missids, missslots, evicted = [], [], [], [], [], []
        for st in range(steps):
            ids, _ = router_topk_softmax(router_logits(n_tok, bias, rng), k)
            r = lay.eval(ids.reshape(-1), is_decode=True)
            assert r["status"] == 0
            ids_all.append(ids)
            slots_all.append(r["slots"].reshape(n_tok, k))
            m = len(r["miss_ids"])
            nmiss.append(m)
            pad = np.full(n_tok * k, -9, np.int32)
            for lst, arr in ((missids, r["miss_ids"]), (missslots, r["miss_slots"]),
                             (evicted, r["evicted"])):
                p = pad.copy()
                p[:m] = arr
                lst.append(p)
        out[f"{name}_meta"] = np.array([E, k, S, pinned, n_tok, steps], np.int32)
        out[f"{name}_ids"] = np.stack(ids_all).astype(np.int32)
        out[f"{name}_slots"] = np.stack(slots_all).astype(np.int32)
        out[f"{name}_nmiss"] = np.array(nmiss, np.int32)
        out[f"{name}_miss_ids"] = np.stack(missids)
        out[f"{name}_miss_slots"] = np.stack(missslots)
        out[f"{name}_evicted"] = np.stack(evicted)
    return out


def router_golden() -> dict:
    from oracle.ref_numpy import router_topk_sigmoid_bias, router_topk_softmax
    from nvmoe_b200.synth import layer_log_bias, router_logits

    rng = np.random.default_rng(3)
    out = {}
    b = layer_log_bias(1, 512, 1.1, seed=3)[0]
    lg = router_logits(32, b, rng)
    ids, w = router_topk_softmax(lg, 10)
    out.update(softmax_logits=lg, softmax_ids=ids, softmax_w=w)
    b2 = rng.standard_normal(288).astype(np.float32) * 0.1
    lg2 = rng.standard_normal((32, 288)).astype(np.float32)
    ids2, w2, _ = router_topk_sigmoid_bias(lg2, 8, b2, True, 2.5)
    out.update(sigmoid_logits=lg2, sigmoid_bias=b2, sigmoid_ids=ids2, sigmoid_w=w2)
    return out


def glm_router_reference(ref: Path) -> dict:
    """Seeded logits routed by the reference's own GLM router (patched_route of
    install_glm5_pruning_patch, nvme-moe-bench/nvme_offload_cache.py:2980-3089), with a stand-in
    Glm5NextSparseBlock whose gate is the identity (so F.linear(hidden, gate) returns the logits
    unchanged) and a top-k override one below the block's top_k (the patched path, not the
    unpatched FreeToken route it falls back to)."""
    import os

    import torch
    _stub_reference_imports()

    class Glm5NextSparseBlock:  # the class the patch wraps (FreeToken, not installed)
        def _route(self, hidden_states):
            raise RuntimeError("the unpatched FreeToken route is not available")

    for name in ("freetoken.models", "freetoken.models.glm5_next", "freetoken.server"):
        sys.modules[name] = types.ModuleType(name)
    moe = types.ModuleType("freetoken.models.glm5_next.moe")
    moe.Glm5NextSparseBlock = Glm5NextSparseBlock
    sys.modules["freetoken.models.glm5_next.moe"] = moe
    args = types.ModuleType("freetoken.server.args")
    args.parse_args = lambda *a, **k: None
    sys.modules["freetoken.server.args"] = args
    sys.path.insert(0, str(ref / "nvme-moe-bench"))
    import nvme_offload_cache as noc  # the reference module
    noc.install_glm5_pruning_patch()
    route = Glm5NextSparseBlock._route
    os.environ.pop("FREETOKEN_ROUTER_MIN_PROB", None)
    os.environ.pop("FREETOKEN_GLM_ROUTER_MIN_PROB", None)
    rng = np.random.default_rng(11)
    out = {}
    for name, E, k, n, norm, scale in (("glm_a", 288, 8, 64, True, 2.5),
                                       ("glm_b", 256, 8, 16, False, 1.0),
                                       ("glm_c", 64, 4, 32, True, 1.0)):
        logits = rng.standard_normal((n, E)).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
        os.environ["FREETOKEN_TOPK_OVERRIDE"] = str(k)
        block = types.SimpleNamespace(
            top_k=k + 1, n_group=1, norm_topk_prob=norm, routed_scaling_factor=scale,
            gate=types.SimpleNamespace(weight=torch.eye(E, dtype=torch.float32)),
            e_score_correction_bias=torch.from_numpy(bias))
        w, ids = route(block, torch.from_numpy(logits))
        out[f"{name}_meta"] = np.array([E, k, n, int(norm)], np.int32)
        out[f"{name}_scale"] = np.array([scale], np.float32)
        out[f"{name}_logits"] = logits
        out[f"{name}_bias"] = bias
        out[f"{name}_ids"] = ids.numpy().astype(np.int32)
        out[f"{name}_w"] = w.numpy().astype(np.float32)
    os.environ.pop("FREETOKEN_TOPK_OVERRIDE", None)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    a = ap.parse_args()
    ref = Path(a.reference)
    (HERE / "slru_traces.json").write_text(json.dumps(slru_traces(ref)))
    np.savez_compressed(HERE / "dequant_golden.npz", **dequant_golden())
    np.savez_compressed(HERE / "remap_traces.npz", **remap_traces())
    np.savez_compressed(HERE / "router_golden.npz", **router_golden())
    np.savez_compressed(HERE / "glm_router_golden.npz", **glm_router_reference(ref))
    for p in sorted(HERE.glob("*.*")):
        print(f"{p.name:24s} {p.stat().st_size:8d} B")


if __name__ == "__main__":
    main()
