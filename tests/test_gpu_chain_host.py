"""GPU: the host-buffer path of the config-4 chain (`EncoderNormChain.step_host`,
chunk groups pipelined over three streams, each group's mel + layers
replayed as one CUDA graph) gives the same bits as the device-resident
step, with and without the graphs, over consecutive steps."""

from __future__ import annotations

import pytest
import torch

from vlasr.pipeline import ChainShape, EncoderNormChain, seeded_pcm

pytestmark = pytest.mark.gpu


def _chain(dev):
    return EncoderNormChain(ChainShape(chunks=6, layers=3), dev, seed=3)


@pytest.mark.parametrize("graphs", [True, False])
def test_step_host_matches_device_step(dev, graphs):
    pcm = torch.from_numpy(seeded_pcm(6, 0, seed=1))
    ref = _chain(dev)
    pcm_dev_ref = pcm.to(dev)
    for _ in range(2):
        ref.step(pcm_dev_ref)
    torch.cuda.synchronize()

    host = _chain(dev)
    pcm_host = pcm.pin_memory()
    mel_host = torch.empty((6, 128, 3000), dtype=torch.float32).pin_memory()
    y_host = torch.empty((host.shape.rows, host.shape.hidden), dtype=torch.bfloat16).pin_memory()
    pcm_dev = torch.empty_like(pcm_dev_ref)
    for _ in range(2):
        mel_host.zero_()
        y_host.zero_()
        host.step_host(pcm_host, mel_host, y_host, pcm_dev, groups=2, graphs=graphs)
    torch.cuda.synchronize()
    assert torch.equal(mel_host, ref.mel.cpu())
    assert torch.equal(y_host, ref.y.cpu())
    assert torch.equal(host.h, ref.h)
    assert torch.equal(host.g_out, ref.g_out)
    if graphs:
        assert len(host._group_graphs) == 3   # host_group_bounds(6, 2): three groups, one buffer
        host.release_graphs()
