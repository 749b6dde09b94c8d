"""The multi-device path on the GPU: shards aligned concurrently from several
host threads give exactly the single-call outputs once gathered."""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from oracle import oracle
from tests.helpers import assert_matches_oracle

pytestmark = pytest.mark.gpu
MODES = ["optimized", "conventional"]
FIELDS = ("labels", "scores", "status", "objective", "stitched", "repair_passes", "repaired_frames",
          "shortcut_stats", "routing_stats", "reuse_stats")


def _same(a, b):
    assert a.lengths == b.lengths
    for name in FIELDS:
        x, y = getattr(a, name).cpu(), getattr(b, name).cpu()
        assert x.shape == y.shape, name
        assert torch.equal(x.view(torch.int32) if x.dtype == torch.float32 else x,
                           y.view(torch.int32) if y.dtype == torch.float32 else y), name


@pytest.mark.parametrize("mode", MODES)
def test_threads_on_one_device_match_one_call(cuda, mode):
    # cfg4's length mix at 1/16 scale: four shards aligned by four threads at
    # once on the same device (each with its own pinned staging ring).
    wl = workloads.config(4, scale=1 / 16)
    es, ts = wl.records()
    host_e = [torch.from_numpy(e).pin_memory() for e in es]
    host_t = [torch.from_numpy(t).pin_memory() for t in ts]
    whole = ffa.align([e.to(cuda) for e in host_e], [t.to(cuda) for t in host_t],
                      blank_id=wl.blank, mode=mode)
    sharded = ffa.align_sharded(host_e, host_t, blank_id=wl.blank, mode=mode, devices=[0, 0, 0, 0])
    assert len(sharded.shards) == 4
    counts = [s.records.size for s in sharded.shards]
    assert sum(counts) == wl.batch and min(counts) > 0
    gathered = sharded.gather(cuda)
    _same(gathered, whole)
    if mode == "conventional":
        assert_matches_oracle(gathered, oracle.align(es, ts, wl.blank))
    assert sharded.status().tolist() == whole.status.cpu().tolist()


def test_sharded_logits_match_one_call(cuda):
    # bf16 logits over three shards on one device: each shard computes its
    # rows' log-sum-exps, and a row's value does not depend on its batch.
    wl = workloads.config(4, scale=1 / 32)
    es, ts = wl.records()
    rng = np.random.default_rng(9)
    logits = [torch.from_numpy(e + rng.uniform(-5, 5, (e.shape[0], 1)).astype(np.float32)).to(torch.bfloat16)
              for e in es]
    targets = [torch.from_numpy(t) for t in ts]
    whole = ffa.align([x.to(cuda) for x in logits], [t.to(cuda) for t in targets], blank_id=wl.blank,
                      from_logits=True)
    sharded = ffa.align_sharded(logits, targets, blank_id=wl.blank, devices=[0, 0, 0], from_logits=True)
    _same(sharded.gather(cuda), whole)


def test_records_stay_on_their_device(cuda):
    wl = workloads.config(0, scale=0.5)
    es, ts = wl.records()
    dev_e = [torch.from_numpy(e).to(cuda) for e in es]
    dev_t = [torch.from_numpy(t).to(cuda) for t in ts]
    sharded = ffa.align_sharded(dev_e, dev_t, blank_id=wl.blank, mode="conventional")
    assert len(sharded.shards) == 1 and sharded.shards[0].device == cuda
    assert np.array_equal(sharded.shards[0].records, np.arange(wl.batch))
    assert_matches_oracle(sharded.gather(cuda), oracle.align(es, ts, wl.blank))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", MODES)
def test_two_devices_match_one_call(cuda, mode):
    wl = workloads.config(1)
    es, ts = wl.records()
    whole = ffa.align([torch.from_numpy(e).to(cuda) for e in es],
                      [torch.from_numpy(t).to(cuda) for t in ts], blank_id=wl.blank, mode=mode)
    sharded = ffa.align_sharded([torch.from_numpy(e).pin_memory() for e in es],
                                [torch.from_numpy(t).pin_memory() for t in ts],
                                blank_id=wl.blank, mode=mode, devices=[0, 1])
    assert {s.device.index for s in sharded.shards} == {0, 1}
    _same(sharded.gather(cuda), whole)
