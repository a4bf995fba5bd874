"""The routing restatement on the CPU: best first, equal logits in ascending expert order, FP32
renormalisation in choice order."""

import torch

from furiosa_opt_models_b200.models import reference as R


def test_ties_go_to_the_lower_expert():
    logits = torch.tensor([[0.5, 1.0, 1.0, -0.0, 0.0, 1.0]]).bfloat16()
    ids, w = R.moe_route(logits, 4, normalize=False)
    assert ids.tolist() == [[1, 2, 5, 0]]
    p = torch.softmax(logits.float(), -1)[0]
    assert torch.allclose(w[0], p[[1, 2, 5, 0]])


def test_signed_zeros_are_equal():
    logits = torch.tensor([[-0.0, 0.0, -1.0]]).bfloat16()
    ids, _ = R.moe_route(logits, 2)
    assert ids.tolist() == [[0, 1]]


def test_normalized_weights_sum_to_one():
    torch.manual_seed(0)
    logits = torch.randn(16, 128).bfloat16()
    _, w = R.moe_route(logits, 8, normalize=True)
    assert torch.allclose(w.sum(-1), torch.ones(16), atol=1e-6)
