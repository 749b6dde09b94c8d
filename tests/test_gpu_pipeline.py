"""AlignStream: host-resident batches aligned with their copies overlapped
give exactly the results of align_packed on device-resident inputs."""
import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from fast_forced_aligner_b200.pipeline import AlignStream

pytestmark = pytest.mark.gpu


def test_stream_of_host_batches_matches_device_calls(cuda):
    batches = [workloads.config(0), workloads.config(1, scale=0.5), workloads.config(3, scale=0.1),
               workloads.config(1, scale=0.25), workloads.config(0, scale=0.5)]
    stream = AlignStream(cuda)
    pending = []
    for k, wl in enumerate(batches):  # every batch in flight before any result is read
        mode = "optimized" if k % 2 == 0 else "conventional"
        e = torch.from_numpy(wl.emissions).pin_memory()
        t = torch.from_numpy(wl.targets).pin_memory()
        pending.append((wl, mode, e, t, stream.submit(e, wl.lengths, t, wl.target_lengths,
                                                       blank_id=wl.blank, mode=mode)))
    for wl, mode, e, t, p in pending:
        got = p.result()
        ref = ffa.align_packed(e.to(cuda), wl.lengths, t.to(cuda), wl.target_lengths,
                               blank_id=wl.blank, mode=mode)
        assert got.lengths == ref.lengths
        assert got.labels.is_pinned() and got.labels.device.type == "cpu"
        assert torch.equal(got.labels, ref.labels.cpu())
        assert torch.equal(got.scores.view(torch.int32), ref.scores.cpu().view(torch.int32))
        assert torch.equal(got.status, ref.status.cpu())
        np.testing.assert_array_equal(got.objective.numpy().view(np.int32),
                                      ref.objective.cpu().numpy().view(np.int32))
        assert [p_.numel() for p_ in got.paths] == list(wl.lengths)


def test_stream_rejects_device_inputs(cuda):
    stream = AlignStream(cuda)
    e = torch.zeros(10, 6, device=cuda)
    with pytest.raises(ValueError, match="host"):
        stream.submit(e, [10], torch.tensor([1]), [1])


def test_stream_of_bf16_logits_matches_device_call(cuda):
    # Host bf16 logits (half the bytes to copy), aligned as their log_softmax.
    wl = workloads.config(1, scale=0.25)
    rng = np.random.default_rng(4)
    x = torch.from_numpy(wl.emissions + rng.uniform(-6, 6, (wl.emissions.shape[0], 1)).astype(np.float32))
    x = x.to(torch.bfloat16).pin_memory()
    t = torch.from_numpy(wl.targets).pin_memory()
    stream = AlignStream("cuda")  # no index: the current device
    assert stream.device == torch.device("cuda", torch.cuda.current_device())
    got = stream.submit(x, wl.lengths, t, wl.target_lengths, blank_id=wl.blank, from_logits=True).result()
    ref = ffa.align_packed(x.to(cuda), wl.lengths, t.to(cuda), wl.target_lengths, blank_id=wl.blank,
                           from_logits=True)
    assert got.lengths == ref.lengths
    assert torch.equal(got.labels, ref.labels.cpu())
    assert torch.equal(got.scores.view(torch.int32), ref.scores.cpu().view(torch.int32))
    assert torch.equal(got.status, ref.status.cpu())
    assert torch.equal(got.objective.view(torch.int32), ref.objective.cpu().view(torch.int32))
