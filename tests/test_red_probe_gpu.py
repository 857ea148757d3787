"""The reduction-throughput probe adds each key tile's ones exactly once."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
def test_red_probe_counts(causal):
    from multi_gpu_flashattention_b200._ext import C
    tiles, heads, D = 6, 3, 64
    dq = torch.zeros(heads, tiles * 128, D, device="cuda")
    C().red_probe(dq, tiles, causal)
    torch.cuda.synchronize()
    exp = torch.tensor([(i + 1) if causal else tiles for i in range(tiles)],
                       dtype=torch.float32, device="cuda")
    exp = exp.repeat_interleave(128).view(1, -1, 1).expand_as(dq)
    assert torch.equal(dq, exp)
