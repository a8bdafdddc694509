"""sample_next_token (LLM.py:63-110) on CPU: greedy, top-k and nucleus masks."""
import torch

from zoomkv_revision_b200.decode_loop import sample_next_token


def test_greedy_below_temperature_floor():
    logits = torch.tensor([[0.1, 3.0, -1.0], [2.0, 0.0, 1.0]])
    assert sample_next_token(logits, 0.0, 0.95, 20).tolist() == [1, 0]


def test_top_k_restricts_the_support():
    g = torch.Generator().manual_seed(0)
    logits = torch.tensor([[5.0, 4.9, 0.0, 0.0, 0.0, 0.0]]).repeat(64, 1)
    out = sample_next_token(logits, 1.0, 0.0, 2, g)
    assert set(out.tolist()) <= {0, 1}


def test_nucleus_keeps_the_token_that_crosses_top_p():
    g = torch.Generator().manual_seed(1)
    p = torch.tensor([0.5, 0.3, 0.15, 0.05])
    logits = p.log().unsqueeze(0).repeat(256, 1)
    out = sample_next_token(logits, 1.0, 0.9, 0, g)
    assert set(out.tolist()) <= {0, 1, 2} and 2 in set(out.tolist())
    out = sample_next_token(logits, 1.0, 0.4, 0, g)
    assert set(out.tolist()) == {0}
