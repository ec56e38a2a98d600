"""Filtered sampling over the top-256 candidate pool (CPU tier): noise identical to the device sampler's,
greedy / top-k=1 reduce to argmax, and with the whole vocabulary inside the pool the draw equals a
full-vocabulary temperature-first top-k/top-p reference."""
import torch

from sglang_neuron_b200.ops.sampling import gumbel_noise_ids, gumbel_noise_ref, sample_filtered


def test_noise_matches_reference():
    ids = torch.tensor([[0, 5, 77, 1000, 201087]])
    for seed, pos in [(0, 0), (1234, 7), (2 ** 40 + 3, 99999)]:
        ref = gumbel_noise_ref(seed, pos, 201088)[ids[0]]
        got = gumbel_noise_ids(torch.tensor([seed]), torch.tensor([pos]), ids)[0]
        assert torch.allclose(got, ref, atol=1e-5)


def _full_reference(logits, t, k, p, seed, pos):
    s = logits.float() / max(t, 1e-6)
    order = s.argsort(descending=True)
    ss = s[order]
    keep = torch.ones_like(ss, dtype=torch.bool)
    if k > 0:
        keep[k:] = False
    probs = torch.softmax(ss.masked_fill(~keep, float("-inf")), -1)
    cum = probs.cumsum(-1) - probs
    keep &= ~(cum >= p)
    keep[0] = True
    ss = ss.masked_fill(~keep, float("-inf"))
    g = gumbel_noise_ref(seed, pos, logits.shape[0])[order]
    return int(order[(ss + g).argmax()])


def test_filtered_matches_full_vocab_reference():
    torch.manual_seed(0)
    V, B = 200, 6
    logits = torch.randn(B, V) * 3
    T = torch.tensor([0.0, 0.7, 1.0, 1.3, 0.5, 2.0])
    K = torch.tensor([0, 0, 5, 1, 50, 0])
    P = torch.tensor([1.0, 0.9, 1.0, 1.0, 0.5, 0.3])
    seeds = torch.arange(B) * 17 + 3
    pos = torch.arange(B) + 40
    got = sample_filtered(logits, T, K, P, seeds, pos)
    for b in range(B):
        if T[b] <= 0:
            assert int(got[b]) == int(logits[b].argmax())
        else:
            assert int(got[b]) == _full_reference(logits[b], float(T[b]), int(K[b]), float(P[b]), int(seeds[b]),
                                                  int(pos[b])), b


def test_sharded_merge_equals_unsharded():
    torch.manual_seed(1)
    V, B = 1000, 4
    logits = torch.randn(B, V)
    T = torch.full((B,), 0.8)
    K = torch.tensor([0, 20, 0, 3])
    P = torch.tensor([0.9, 1.0, 0.5, 1.0])
    seeds, pos = torch.arange(B) + 5, torch.arange(B) + 9
    whole = sample_filtered(logits, T, K, P, seeds, pos)
    halves = [logits[:, :500], logits[:, 500:]]

    def merge(vals, ids):  # emulate the gather of the other shard's pool
        other = 1 - merge.shard
        ov, oi = halves[other].float().topk(256, dim=-1)
        oi = oi + 500 * other
        av, ai = torch.cat([vals, ov], 1), torch.cat([ids, oi], 1)
        mv, sel = av.topk(256, dim=-1)
        return mv, ai.gather(1, sel)
    for shard in (0, 1):
        merge.shard = shard
        got = sample_filtered(halves[shard], T, K, P, seeds, pos, vocab_offset=500 * shard, valid_vocab=500,
                              merge=merge)
        assert torch.equal(got, whole)
