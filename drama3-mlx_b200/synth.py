"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved; the reference publishes none
for this path). Generated on the device with torch's generator, so a seed
reproduces a batch on the same software stack; parity tests copy the rows they
check to the host.

  C1  f32  [1, 4097]      N(0, 3), one semantic logit (1..4096) +6
  C2  bf16 [256, 4097]    N(0, 2); 1-5 peaked tokens +U[4, 10]; eos (col 0) N(-4, 1)
  C4  bf16 [rows, 1024]   N(0, 2.5) + Zipf(s=1.1) bias over a seeded permutation
  C5  f32  [65536, 4097]  N(0, 3); per-row T ~ U[0.5, 1.2], top_p ~ U[0.5, 1.0],
                          top_k ~ U{1..64}; per-row seeds
("N(mu, s)" has standard deviation s.)
"""

from __future__ import annotations

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def c1_rows(n: int, seed: int, device="cuda", V: int = 4097) -> torch.Tensor:
    g = _gen(seed, device)
    x = torch.randn(n, V, generator=g, device=device) * 3.0
    idx = torch.randint(1, V, (n,), generator=g, device=device)
    x[torch.arange(n, device=device), idx] += 6.0
    return x


def c2_logits(N: int = 256, seed: int = 0, device="cuda", V: int = 4097) -> torch.Tensor:
    g = _gen(seed, device)
    x = torch.randn(N, V, generator=g, device=device) * 2.0
    n_peaks = torch.randint(1, 6, (N,), generator=g, device=device)
    pos = torch.randint(1, V, (N, 5), generator=g, device=device)
    boost = torch.rand(N, 5, generator=g, device=device) * 6.0 + 4.0
    boost = boost * (torch.arange(5, device=device)[None, :] < n_peaks[:, None])
    x.scatter_add_(1, pos, boost)
    x[:, 0] = torch.randn(N, generator=g, device=device) - 4.0
    return x.to(torch.bfloat16)


def zipf_bias(V: int, seed: int, s: float = 1.1, device="cuda") -> torch.Tensor:
    """log-probability bias of a Zipf(s) law over a seeded permutation of V ids."""
    g = _gen(seed, device)
    ranks = torch.arange(1, V + 1, device=device, dtype=torch.float64)
    logp = -s * torch.log(ranks)
    logp = logp - torch.logsumexp(logp, 0)
    perm = torch.randperm(V, generator=g, device=device)
    out = torch.empty(V, device=device, dtype=torch.float32)
    out[perm] = logp.float()
    return out


def c4_logits(rows: int, seed: int, device="cuda", V: int = 1024,
              bias: torch.Tensor | None = None) -> torch.Tensor:
    g = _gen(seed, device)
    if bias is None:
        bias = zipf_bias(V, seed ^ 0x5EED, device=device)
    x = torch.randn(rows, V, generator=g, device=device) * 2.5 + bias[None, :]
    return x.to(torch.bfloat16)


def c3_inputs(B: int, seed: int = 0, device="cuda", V: int = 4097, D: int = 2048):
    """(h bf16 [B, D] ~ N(0, 1), W bf16 [V, D] ~ N(0, 0.02)): the hidden states
    and the restricted lm_head weight of the fused-prologue config."""
    g = _gen(seed, device)
    h = torch.randn(B, D, generator=g, device=device).to(torch.bfloat16)
    W = (torch.randn(V, D, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return h, W


def c5_batch(N: int = 65536, seed: int = 0, device="cuda", V: int = 4097):
    """(logits f32 [N, V], temperature [N], top_p [N], top_k int32 [N], seeds int64 [N])."""
    g = _gen(seed, device)
    x = torch.randn(N, V, generator=g, device=device) * 3.0
    T = torch.rand(N, generator=g, device=device) * 0.7 + 0.5
    p = torch.rand(N, generator=g, device=device) * 0.5 + 0.5
    k = torch.randint(1, 65, (N,), generator=g, device=device, dtype=torch.int32)
    seeds = torch.arange(N, device=device, dtype=torch.int64) + seed * 1_000_003
    return x, T, p, k, seeds


def to_host_logits(x: torch.Tensor):
    """Host copy for the oracle: float32 as is, bfloat16 as raw uint16 bits."""
    if x.dtype == torch.bfloat16:
        return x.contiguous().view(torch.int16).cpu().numpy().view("uint16")
    return x.float().contiguous().cpu().numpy()
