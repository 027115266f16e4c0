"""Same-box PyTorch baseline of the Llama decode step (``bench.py --impl torch``).

The decode step written with stock PyTorch only:
- cuBLAS GEMMs through ``F.linear``;
- ``F.rms_norm``, SiLU and RoPE as torch ops;
- KV writes by index assignment;
- ``F.scaled_dot_product_attention`` with GQA over a contiguous KV cache, masked to each row's length;
- argmax sampling.

It is captured with ``torch.cuda.graph`` at the engine's decode batch sizes into one shared pool,
largest first, as engines do. The model, batch, prompt length, weight init and graph sizes are the
ones the foundry arm of bench.py uses. None of this package's kernels, engine or persistence run here.

What the timed loop measures is the same as the foundry arm: K replays of the
batch-B graph, each feeding its sampled tokens back and advancing the
positions on the device. The KV cache is filled with random values of the prompt length
instead of a prefill; decode cost depends on the lengths, not on the cached values.
Attention reads every cache slot up to the longest length of the batch (the
mask covers the rest), which in this benchmark (equal-length prompts) is the
same length the paged kernels read.
"""

from __future__ import annotations

import math
import time

import torch
import torch.nn.functional as F

from ..models import config_by_name


class TorchLlama:
    """bf16 weights N(0, 0.02), norms 1, contiguous KV cache [L][B, n_kv, S, d]."""

    def __init__(self, cfg, max_batch: int, max_len: int, device="cuda", seed: int = 0):
        self.cfg, self.max_batch, self.max_len = cfg, max_batch, max_len
        h, d = cfg.hidden, cfg.head_dim
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def mat(o, i):
            return torch.randn(o, i, device=device, dtype=bf, generator=g) * cfg.init_std

        self.embed = mat(cfg.vocab, h)
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "attn_norm": torch.ones(h, device=device, dtype=bf), "qkv": mat(cfg.qkv_dim, h),
                "o": mat(h, cfg.n_q * d), "mlp_norm": torch.ones(h, device=device, dtype=bf),
                "gate_up": mat(2 * cfg.inter, h), "down": mat(h, cfg.inter),
            })
        self.final_norm = torch.ones(h, device=device, dtype=bf)
        self.lm_head = mat(cfg.vocab, h)
        shape = (max_batch, cfg.n_kv, max_len, d)
        self.k_cache = [torch.randn(shape, device=device, dtype=bf, generator=g) for _ in range(cfg.layers)]
        self.v_cache = [torch.randn(shape, device=device, dtype=bf, generator=g) for _ in range(cfg.layers)]
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))
        ang = torch.arange(max_len, device=device, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos, self.sin = ang.cos(), ang.sin()  # [S, d/2]
        self.slots = torch.arange(max_len, device=device)
        # static step inputs / outputs (graphs read and write these)
        self.tokens = torch.zeros(max_batch, dtype=torch.long, device=device)
        self.positions = torch.zeros(max_batch, dtype=torch.long, device=device)
        self.next_tokens = torch.zeros(max_batch, dtype=torch.long, device=device)
        self.rows = torch.arange(max_batch, device=device)

    def _rope(self, x, pos):  # x [b, heads, d], rotate-half layout
        c, s = self.cos[pos][:, None, :], self.sin[pos][:, None, :]
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)

    def step(self, b: int) -> None:
        """One decode step for rows [:b]: writes next_tokens, advances positions."""
        cfg = self.cfg
        nq, nkv, d = cfg.n_q, cfg.n_kv, cfg.head_dim
        tok, pos, rows = self.tokens[:b], self.positions[:b], self.rows[:b]
        x = F.embedding(tok, self.embed)
        mask = (self.slots[None, :] <= pos[:, None])[:, None, None, :]  # [b, 1, 1, S]
        for li, lw in enumerate(self.layers):
            hn = F.rms_norm(x, (cfg.hidden,), lw["attn_norm"], cfg.eps)
            qkv = F.linear(hn, lw["qkv"])
            q = self._rope(qkv[:, : nq * d].view(b, nq, d), pos)
            k = self._rope(qkv[:, nq * d: (nq + nkv) * d].view(b, nkv, d), pos)
            v = qkv[:, (nq + nkv) * d:].view(b, nkv, d)
            kc, vc = self.k_cache[li], self.v_cache[li]
            kc[rows, :, pos] = k
            vc[rows, :, pos] = v
            o = F.scaled_dot_product_attention(q[:, :, None, :], kc[:b], vc[:b], attn_mask=mask,
                                               scale=1.0 / math.sqrt(d), enable_gqa=True)
            x = x + F.linear(o.reshape(b, nq * d), lw["o"])
            hn = F.rms_norm(x, (cfg.hidden,), lw["mlp_norm"], cfg.eps)
            gate, up = F.linear(hn, lw["gate_up"]).chunk(2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, lw["down"])
        logits = F.linear(F.rms_norm(x, (cfg.hidden,), self.final_norm, cfg.eps), self.lm_head)
        self.next_tokens[:b].copy_(logits.argmax(-1))
        self.positions[:b].add_(1)


def run(model: str, batch: int, prompt_len: int, gen: int, steps: int, warmup: int, graph_sizes: list[int],
        device: int = 0) -> dict:
    """Captures the graphs, times ``steps`` replays of the batch graph; device times in ms."""
    cfg = config_by_name(model)
    if getattr(cfg, "arch", "llama") != "llama":
        raise ValueError(f"the PyTorch baseline covers the dense Llama family, not {model}")
    torch.cuda.set_device(device)
    max_batch = max(max(graph_sizes), batch)
    net = TorchLlama(cfg, max_batch, prompt_len + gen)
    net.positions.fill_(prompt_len)
    net.tokens.random_(0, cfg.vocab)
    # eager warm-up of every size (cuBLAS heuristics, lazy module loads) outside capture
    for bs in sorted(set(graph_sizes + [batch]), reverse=True):
        net.step(bs)
        net.positions.fill_(prompt_len)
    torch.cuda.synchronize()
    pool = torch.cuda.graph_pool_handle()
    graphs = {}
    t0 = time.perf_counter()
    for bs in sorted(set(graph_sizes + [batch]), reverse=True):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            net.step(bs)
        graphs[bs] = g
    torch.cuda.synchronize()
    capture_s = time.perf_counter() - t0
    net.positions.fill_(prompt_len)
    g = graphs[batch]
    for _ in range(warmup):
        g.replay()
        net.tokens[:batch].copy_(net.next_tokens[:batch])
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        g.replay()
        net.tokens[:batch].copy_(net.next_tokens[:batch])
    end.record()
    torch.cuda.synchronize()
    dev_ms = start.elapsed_time(end)
    assert int(net.positions[0]) <= prompt_len + gen, "ran past the cache"
    n_graphs = len(graphs)
    del graphs, g
    return {"dev_ms": dev_ms, "capture_s": capture_s, "num_graphs": n_graphs,
            "kernels_note": "cuBLAS GEMMs, torch SDPA and elementwise kernels (none of this package's)"}



def _main(argv=None) -> int:
    """One eager decode step of the baseline (for a kernel launch list):
    python -m foundry_b200.runner.torch_baseline --model llama-3-8b@2l --batch 256 --ctx 512"""
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b@2l")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=512)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args(argv)
    cfg = config_by_name(a.model)
    net = TorchLlama(cfg, a.batch, a.ctx + a.warmup + 2)
    net.tokens.random_(0, cfg.vocab)
    net.positions.fill_(a.ctx)
    for _ in range(a.warmup):
        net.step(a.batch)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    net.step(a.batch)
    end.record()
    torch.cuda.synchronize()
    print({"eager_step_ms": start.elapsed_time(end), "layers": cfg.layers, "batch": a.batch})
    return 0


__all__ = ["TorchLlama", "run"]


if __name__ == "__main__":
    raise SystemExit(_main())
