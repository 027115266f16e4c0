"""The PyTorch baseline of bench.py (foundry_b200/runner/torch_baseline.py)
computes the real model: token-by-token decode steps of a small Llama on the
CPU reproduce the fp32 reference forward's greedy tokens, so its timing is
of the same work as the foundry arm's."""

import torch

from foundry_b200.models.llama import reference_forward, tiny
from foundry_b200.runner.torch_baseline import TorchLlama


def test_decode_steps_match_reference_forward():
    cfg = tiny(layers=2, vocab=512)
    net = TorchLlama(cfg, max_batch=2, max_len=24, device="cpu", seed=3)
    # the baseline's tables in the reference's [pos, d/2, (cos, sin)] layout
    cos_sin = torch.stack([net.cos, net.sin], dim=-1)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab, (7,), generator=g), torch.randint(0, cfg.vocab, (7,), generator=g)]
    net.positions.zero_()
    outs = [[], []]
    for t in range(12):
        for r in range(2):
            net.tokens[r] = prompts[r][t] if t < 7 else outs[r][-1]
        net.step(2)
        if t >= 6:
            for r in range(2):
                outs[r].append(int(net.next_tokens[r]))
    checked = 0
    for r in range(2):
        seq = torch.cat([prompts[r], torch.tensor(outs[r][:-1])])
        logits = reference_forward(cfg, net, seq, cos_sin)
        for j in range(len(outs[r])):
            top2 = logits[6 + j].topk(2)
            if top2.values[0] - top2.values[1] > 0.05:  # bf16 activations vs fp32 reference
                assert outs[r][j] == int(top2.indices[0]), (r, j, outs[r], top2)
                checked += 1
    assert checked >= 6, checked
