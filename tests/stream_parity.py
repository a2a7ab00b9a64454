"""Greedy-stream comparison used by the end-to-end GPU tests.

Two implementations that round differently cannot be required to produce the same greedy token at
a step whose top-2 logit margin is smaller than the logit noise that rounding produces: at such a
step the argmax is not determined by the math. The reference's own paths show this. Its literal
attention (bf16 scores) and the fp32-softmax parity oracle differ only in the attention rounding,
yet their logits differ by up to ~0.25 at the full 36-layer Qwen3-4B depth, and the oracle's bf16
logits have exact top-2 ties at some steps. So the comparison is:

* ``band`` = the largest logit difference between the reference's literal path and the fp32
  oracle, teacher-forced along the oracle's stream: the reference's own numerical noise.
* A step is *decided* when the oracle's top-2 margin exceeds ``2 * band``. At every decided step
  the engine's argmax must equal the oracle's (and the reference's). This is not implied by the
  engine's own noise: an engine noisier than the reference would fail it.
* The free-running engine stream must equal the oracle's stream up to the first undecided step.
* The engine's logit noise must not exceed the reference's by more than a stated factor.

``compare`` returns every number (steps, decided count, undecided steps with their margins, first
divergences of the free-running streams) so the tests can print and assert them.
"""

from __future__ import annotations

import torch


def teacher_forced(runner, prompt: torch.Tensor, tokens: list[int]) -> list[torch.Tensor]:
    """Logits of ``runner`` at every step of ``tokens`` (prefill, then one decode per token)."""
    out = [runner.prefill(prompt).float().clone()]
    pos = int(prompt.shape[0])
    for t in tokens[:-1]:
        out.append(runner.decode(t, pos).float().clone())
        pos += 1
    return out


def first_divergence(a: list[int], b: list[int]) -> int | None:
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def compare(oracle_stream, oracle_logits, ref_logits, ours_logits, ours_stream, ref_stream=None):
    margins = []
    for lg in oracle_logits:
        t2 = lg.flatten().topk(2).values
        margins.append((t2[0] - t2[1]).item())
    d_ref = [(a - b).abs().max().item() for a, b in zip(ref_logits, oracle_logits)]
    d_ours = [(a - b).abs().max().item() for a, b in zip(ours_logits, oracle_logits)]
    band = max(d_ref)
    decided = [i for i, m in enumerate(margins) if m > 2 * band]
    undecided = [i for i, m in enumerate(margins) if m <= 2 * band]
    arg = lambda lst: [int(x.flatten().argmax().item()) for x in lst]  # noqa: E731
    a_o, a_r, a_s = arg(oracle_logits), arg(ref_logits), arg(ours_logits)
    first_undecided = undecided[0] if undecided else len(margins)
    return {
        "steps": len(margins),
        "band": band,
        "max_d_ours": max(d_ours), "max_d_ref": max(d_ref),
        "mean_d_ours": sum(d_ours) / len(d_ours), "mean_d_ref": sum(d_ref) / len(d_ref),
        "decided": len(decided),
        "undecided_steps": undecided,
        "undecided_margins": [round(margins[i], 5) for i in undecided],
        "exact_ties": sum(1 for m in margins if m == 0.0),
        "decided_mismatch_ours": [i for i in decided if a_s[i] != a_o[i]],
        "decided_mismatch_ref": [i for i in decided if a_r[i] != a_o[i]],
        "forced_flips_ours": [i for i in range(len(margins)) if a_s[i] != a_o[i]],
        "forced_flips_ref": [i for i in range(len(margins)) if a_r[i] != a_o[i]],
        "first_undecided": first_undecided,
        "first_divergence_ours": first_divergence(ours_stream, oracle_stream),
        "first_divergence_ref": None if ref_stream is None else first_divergence(ref_stream, oracle_stream),
    }


def assert_stream_parity(res: dict, noise_factor: float = 1.25) -> None:
    assert not res["decided_mismatch_ours"], res
    assert res["max_d_ours"] <= noise_factor * res["max_d_ref"] + 1e-3, res
    assert res["mean_d_ours"] <= noise_factor * res["mean_d_ref"] + 1e-3, res
    div = res["first_divergence_ours"]
    assert div is None or div >= res["first_undecided"], res
