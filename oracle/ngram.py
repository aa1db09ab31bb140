"""n-gram (prompt lookup) proposer, restated (TEST INFRASTRUCTURE).

Follows ``NgramProposer.propose`` (nanoengine/src/nanoengine/engine/speculative/proposers.py:44-57):

* try n = ``max_ngram`` down to ``min_ngram`` (skipping n when ``len(history) <= n``);
* the suffix is the last n tokens of the whole history (prompt + generated);
* scan start positions from ``len - n - 1`` down to 0, so the most recent earlier match wins;
* propose ``history[start + n : start + n + k]`` (truncated at the end of the history);
* an empty slice keeps scanning (it cannot happen for k >= 1, since start + n <= len - 1);
* no match at any n -> no guesses.
"""

from __future__ import annotations

import numpy as np


def propose(history: list[int], num_tokens: int, max_ngram: int, min_ngram: int = 1) -> list[int]:
    """Pure-Python loops, line for line with the reference semantics (small cases)."""
    for n in range(max_ngram, min_ngram - 1, -1):
        if len(history) <= n:
            continue
        suffix = history[-n:]
        for start in range(len(history) - n - 1, -1, -1):
            if history[start : start + n] == suffix:
                follow = start + n
                guesses = history[follow : follow + num_tokens]
                if guesses:
                    return list(guesses)
    return []


def propose_numpy(history, num_tokens: int, max_ngram: int, min_ngram: int = 1) -> list[int]:
    """Vectorised restatement for long histories (same result as :func:`propose`)."""
    h = np.asarray(history, dtype=np.int64)
    length = h.shape[0]
    if num_tokens <= 0:
        return []
    for n in range(max_ngram, min_ngram - 1, -1):
        if length <= n:
            continue
        starts = length - n  # candidate starts 0 .. length-n-1
        match = np.ones(starts, dtype=bool)
        for j in range(n):
            match &= h[j : j + starts] == h[length - n + j]
        hits = np.nonzero(match)[0]
        if hits.size:
            follow = int(hits[-1]) + n
            return h[follow : follow + num_tokens].tolist()
    return []
