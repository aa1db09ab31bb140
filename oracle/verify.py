"""Token probabilities and speculative verification, restated (TEST INFRASTRUCTURE).

Follows (paths relative to ``nanoengine/src/nanoengine``):

* ``apply_top_p``                 engine/sampling.py:21-27
* ``compute_token_probabilities`` engine/sampling.py:30-38
* ``pick_token``                  engine/speculative/verifier.py:21-24
* ``verify_proposal``             engine/speculative/verifier.py:27-60

The reference draws its random numbers from a ``torch.Generator`` (``torch.rand`` in
``verify_proposal`` and ``torch.multinomial`` in ``sample_from_probabilities``). Here every draw is
taken from an injected iterator of float uniforms instead, in the same data-dependent order:

* one uniform per guess whose acceptance ``a`` satisfies ``0 < a < 1`` (compared ``u < a``);
* one uniform for the correction / bonus token when the temperature is not zero, turned into a
  token by inverse-CDF sampling: the first index whose float64 prefix sum is ``> u * total``.

``tests/golden/make_golden.py`` runs the unmodified reference ``verify_proposal`` with the same
injection (``torch.rand`` and ``sample_from_probabilities`` patched) to pin this restatement.
"""

from __future__ import annotations

import numpy as np
import torch
from torch.nn import functional

GREEDY_TEMPERATURE = 0.0


def apply_top_p(probabilities: torch.Tensor, top_p: float, stable: bool = False) -> torch.Tensor:
    """engine/sampling.py:21-27: keep tokens whose sorted mass-before is < top_p, renormalise.

    ``stable=False`` is the reference's own (unstable) ``torch.sort``; ``stable=True`` orders equal
    probabilities by ascending token id, the convention of the CUDA kernels (which tokens of a tie
    group straddling the cut survive is otherwise implementation-defined)."""
    sorted_p, order = torch.sort(probabilities, descending=True, stable=stable)
    before = torch.cumsum(sorted_p, dim=-1) - sorted_p
    sorted_p[before >= top_p] = 0.0
    kept = torch.zeros_like(probabilities).scatter(-1, order, sorted_p)
    return kept / kept.sum(dim=-1, keepdim=True)


def token_probabilities(logits: torch.Tensor, temperature: float, top_p: float, stable: bool = False) -> torch.Tensor:
    """engine/sampling.py:30-38 (one-hot argmax when greedy)."""
    if temperature == GREEDY_TEMPERATURE:
        return functional.one_hot(torch.argmax(logits, dim=-1), logits.shape[-1]).float()
    probabilities = torch.softmax(logits.float() / temperature, dim=-1)
    if top_p < 1.0:
        probabilities = apply_top_p(probabilities, top_p, stable)
    return probabilities


def inverse_cdf(probabilities: torch.Tensor, u: float) -> int:
    """The injected replacement of ``torch.multinomial(p, 1)``: first i with prefix64[i] > u*total."""
    prefix = np.cumsum(probabilities.detach().double().cpu().numpy())
    return int(np.searchsorted(prefix, u * prefix[-1], side="right"))


def pick_token(probabilities: torch.Tensor, temperature: float, uniforms) -> int:
    """engine/speculative/verifier.py:21-24."""
    if temperature == GREEDY_TEMPERATURE:
        return int(torch.argmax(probabilities).item())
    return inverse_cdf(probabilities, next(uniforms))


def verify_proposal(
    guesses: list[int],
    draft_probabilities: torch.Tensor | None,
    target_logits: torch.Tensor,
    temperature: float,
    top_p: float,
    uniforms,
    stable: bool = False,
) -> list[int]:
    """engine/speculative/verifier.py:27-60: kept guesses plus one target token."""
    target = token_probabilities(target_logits, temperature, top_p, stable)
    vocab = target.shape[-1]
    kept: list[int] = []
    for index, guess in enumerate(guesses):
        if draft_probabilities is None:
            draft = functional.one_hot(torch.tensor(guess), vocab).float()
        else:
            draft = draft_probabilities[index].float()
        acceptance = (target[index, guess] / draft[guess].clamp(min=1e-12)).clamp(max=1.0).item()
        if acceptance >= 1.0 or (acceptance > 0.0 and next(uniforms) < acceptance):
            kept.append(guess)
            continue
        residual = (target[index] - draft).clamp(min=0.0)
        if residual.sum() <= 0:
            residual = target[index]
        residual = residual / residual.sum()
        return [*kept, pick_token(residual, temperature, uniforms)]
    return [*kept, pick_token(target[len(guesses)], temperature, uniforms)]
