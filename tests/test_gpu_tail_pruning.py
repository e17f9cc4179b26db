"""(f)3 tail pruning on the device (nvmoe_prune_tail, scripts/moe_cache_probe.cpp:523-625)
against the oracle's restatement, which the CPU tests pin to the reference's own block: ids,
weights and decode counters bit for bit over random residencies, host tiers, thresholds and
batch sizes, with rows read through a row stride wider than top_k."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from oracle import ref_numpy as R
from tests.test_prune_cpu import _case

pytestmark = pytest.mark.gpu


def test_prune_tail_kernel_matches_oracle(cuda_device):
    pruned_any = 0
    for seed in range(600, 720):
        (ids, w, sor, hs, ris), cfg = _case(seed)
        n, k = ids.shape
        table = ops.SlotTableGPU(len(sor), len(ris), cuda_device)
        table.slot_of_real.copy_(torch.from_numpy(sor))
        table.real_in_slot.copy_(torch.from_numpy(ris))
        wide_i = torch.full((n, k + 3), -5, dtype=torch.int32, device=cuda_device)
        wide_w = torch.full((n, k + 3), -2.0, dtype=torch.float32, device=cuda_device)
        wide_i[:, 1:1 + k] = torch.from_numpy(ids).to(cuda_device)
        wide_w[:, 1:1 + k] = torch.from_numpy(w).to(cuda_device)
        cnt = torch.zeros(2, dtype=torch.int32, device=cuda_device)
        ops.prune_tail(wide_i[:, 1:1 + k], wide_w[:, 1:1 + k], table, cfg["nvme_thresh"],
                       cfg["host_thresh"], cfg["min_keep"], cfg["min_mass"],
                       host_slot_of_real=None if hs is None else torch.from_numpy(hs).to(cuda_device),
                       is_decode=cfg["is_decode"], pruned=cnt)
        ri, rw, pn, ph = R.prune_tail(ids, w, sor, hs, ris, **cfg)
        gi, gw = wide_i.cpu().numpy(), wide_w.cpu().numpy()
        np.testing.assert_array_equal(gi[:, 1:1 + k], ri, err_msg=str(seed))
        assert gw[:, 1:1 + k].tobytes() == rw.tobytes(), seed
        assert (gi[:, 0] == -5).all() and (gi[:, 1 + k:] == -5).all()
        assert (gw[:, 0] == -2).all() and (gw[:, 1 + k:] == -2).all()
        assert tuple(cnt.cpu().tolist()) == (pn, ph), seed
        pruned_any += pn + ph
    assert pruned_any > 20
