"""Near-tie bookkeeping shared by the GPU parity tests.

A token whose 8th and 9th router logits lie closer together than the GPU-vs-oracle logit error can legitimately
route to a different expert on the GPU than in the oracle, so its outputs are left out of the value comparisons.
Every test that leaves tokens out goes through `keep_stable`, which requires at least MIN_KEPT of the tokens to be
compared and records how many were left out and the smallest 8th/9th margin seen; the session summary
(tests/conftest.py) prints that record.
"""
import os

import numpy as np

MIN_KEPT = 0.9
EXCLUDED = []  # (test id, tokens left out, tokens, smallest 8th/9th margin)


def _current_test():
    return os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]


def topk_margin(logits, topk):
    """The 8th/9th (k-th / k+1-th) logit margin of each row."""
    srt = np.sort(np.asarray(logits), axis=1)[:, ::-1]
    if srt.shape[1] <= topk:
        return np.full(srt.shape[0], np.inf)
    return srt[:, topk - 1] - srt[:, topk]


def keep_stable(ok, margin):
    """Records the left-out tokens of the calling test and asserts that at least MIN_KEPT are compared."""
    ok = np.asarray(ok, dtype=bool)
    margin = np.asarray(margin, dtype=np.float64)
    n_out = int((~ok).sum())
    EXCLUDED.append((_current_test(), n_out, int(ok.size), float(margin.min()) if margin.size else float("inf")))
    assert ok.mean() >= MIN_KEPT, (f"{n_out} of {ok.size} tokens sit within the logit error of an 8th/9th routing tie "
                                   f"(smallest margin {margin.min():.3g}); at most {1 - MIN_KEPT:.0%} may be left out")
    return ok
