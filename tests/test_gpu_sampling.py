"""The sampling kernel (``sample_pass``) against the torch sampler (the CPU oracle).

On the GPU the sampler's per-element work is one kernel pass over the vocabulary shard;
it must draw the tokens the torch implementation draws (same hash noise, same masks; a
rare near-tie may flip under different float rounding), follow the truncated softmax,
verify drafts exactly, and give the same tokens when the vocabulary is split over ranks.
"""
import numpy as np
import pytest
import torch

from oscar_b200.ops import sampling as S

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rows(n, temperature, top_k, top_p, seed, pos, draft, dev="cpu", truncated=True):
    return S.SampleRows(temperature.float().to(dev), top_k.int().to(dev), top_p.float().to(dev), seed.int().to(dev),
                        pos.int().to(dev), draft.int().to(dev), truncated)


def _mixed(n, V, g):
    temps = torch.tensor([0.0, 0.7, 1.0, 1.5])[torch.arange(n) % 4]
    top_k = torch.tensor([0, 0, 7, 200])[torch.arange(n) % 4]
    top_p = torch.tensor([1.0, 0.85, 1.0, 0.6])[torch.arange(n) % 4]
    seed = torch.arange(n) * 31 + 5
    pos = torch.arange(n) + 100
    draft = torch.randint(-1, V, (n,), generator=g)
    return temps, top_k, top_p, seed, pos, draft


@pytest.mark.parametrize("V,begin", [(65536, 0), (70001, 1000)])
def test_kernel_draws_the_torch_tokens(V, begin):
    g = torch.Generator().manual_seed(V)
    n = 96
    logits = (torch.randn(n, V, generator=g) * 3).to(torch.bfloat16)
    temps, top_k, top_p, seed, pos, draft = _mixed(n, V, g)
    draft = torch.where(draft >= 0, draft + begin, draft)
    want = S.sample(logits, begin, _rows(n, temps, top_k, top_p, seed, pos, draft))
    got = S.sample(logits.to(DEV), begin, _rows(n, temps, top_k, top_p, seed, pos, draft, DEV)).cpu()
    greedy = temps == 0
    assert torch.equal(got[greedy], want[greedy])
    assert (got == want).float().mean().item() >= 0.97


def test_untruncated_steps_skip_the_threshold_phase():
    """Rows without top-k / top-p give the same tokens with and without phase 1."""
    g = torch.Generator().manual_seed(11)
    n, V = 40, 50000
    logits = (torch.randn(n, V, generator=g) * 2).to(torch.bfloat16).to(DEV)
    temps = torch.tensor([0.0, 0.8] * 20)
    args = (temps, torch.zeros(n), torch.ones(n), torch.arange(n) + 3, torch.arange(n),
            torch.randint(-1, V, (n,), generator=g))
    a = S.sample(logits, 0, _rows(n, *args, dev=DEV, truncated=True))
    b = S.sample(logits, 0, _rows(n, *args, dev=DEV, truncated=False))
    assert torch.equal(a, b)


@pytest.mark.parametrize("params,draft", [(S.SamplingParams(temperature=1.0), -1),
                                          (S.SamplingParams(temperature=0.8, top_k=8), 1),
                                          (S.SamplingParams(temperature=1.0, top_p=0.9), 0)])
def test_kernel_samples_follow_the_truncated_distribution(params, draft):
    base = torch.randn(64, generator=torch.Generator().manual_seed(3)) * 2.0
    base = base.to(torch.bfloat16).float()
    N, V = 40000, 64
    logits = base.unsqueeze(0).expand(N, V).contiguous().to(torch.bfloat16).to(DEV)
    d = -1 if draft < 0 else int(torch.argsort(base, descending=True)[draft])
    rows = _rows(N, torch.full((N,), params.temperature), torch.full((N,), params.top_k),
                 torch.full((N,), params.top_p), torch.full((N,), 7), torch.arange(N), torch.full((N,), d), DEV,
                 truncated=params.top_k > 0 or params.top_p < 1)
    tok = S.sample(logits, 0, rows).cpu()
    p = S.probabilities(base, params).numpy()
    f = np.bincount(tok.numpy(), minlength=V) / N
    assert np.all(f[p == 0] == 0), "sampled a truncated token"
    assert 0.5 * np.abs(f - p).sum() < 0.02
    if d >= 0:
        assert abs(f[d] - p[d]) < 0.01  # acceptance rate = p(d)


def test_vocab_split_over_ranks_draws_the_same_tokens():
    g = torch.Generator().manual_seed(5)
    n, V = 48, 30000
    logits = (torch.randn(n, V, generator=g) * 3).to(torch.bfloat16).to(DEV)
    temps, _, _, seed, pos, draft = _mixed(n, V, g)
    rows = _rows(n, temps, torch.zeros(n), torch.ones(n), seed, pos, draft, DEV, truncated=False)
    tau = torch.full((n,), float("-inf"), device=DEV)
    want = S._combine_cuda(S._pass_cuda(logits, 0, rows, tau).unsqueeze(0), rows)
    for cut in (8192, 12345, 29999):
        parts = torch.stack([S._pass_cuda(logits[:, :cut].contiguous(), 0, rows, tau),
                             S._pass_cuda(logits[:, cut:].contiguous(), cut, rows, tau)])
        assert torch.equal(S._combine_cuda(parts, rows), want), cut
