"""Nucleus (top-p) masking of the sampler against a direct restatement."""
import torch

from quantized_flash_communication_b200.models.sampling import top_p_mask


def _direct(logits, inv_temp, top_p):
    out = torch.full_like(logits, float("-inf"))
    for r in range(logits.shape[0]):
        p = torch.softmax(logits[r] * inv_temp, -1)
        order = sorted(range(p.numel()), key=lambda i: -float(p[i]))
        acc = 0.0
        for i in order:  # keep tokens until the kept mass reaches top_p
            out[r, i] = logits[r, i]
            acc += float(p[i])
            if acc >= top_p:
                break
    return out


def test_top_p_mask_matches_direct_definition():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(6, 50, generator=g) * 3
    for top_p in (0.05, 0.5, 0.9, 0.999):
        got = top_p_mask(logits, 1 / 0.7, top_p)
        ref = _direct(logits, 1 / 0.7, top_p)
        assert torch.equal(torch.isinf(got), torch.isinf(ref)), top_p
        assert torch.equal(got[~torch.isinf(got)], ref[~torch.isinf(ref)])


def test_top_p_keeps_at_least_the_best_token():
    logits = torch.tensor([[10.0, 0.0, -1.0]])
    got = top_p_mask(logits, 1.0, 1e-6)
    assert got[0, 0] == 10.0 and torch.isinf(got[0, 1:]).all()
