"""Generate golden draft/replay vectors from the reference's own Python tool.

Run where the reference tree is checked out, with its path as the only
argument: python tests/golden/make_golden.py <reference checkout>.  It imports
cpu-lab/moss_ngram_audit.py (draft(), replay()) from the reference and records
its outputs on seeded histories; the vectors are committed as
tests/golden/ngram_draft.json and tests/golden/ngram_replay.json so the tests
never need the reference at run time.
"""
import json
import os
import random
import sys


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    ref = sys.argv[1]
    sys.path.insert(0, os.path.join(ref, "cpu-lab"))
    import moss_ngram_audit as audit  # noqa: E402  (the reference's replay tool)

    rng = random.Random(20261201)
    draft_cases = []
    params = [(4, 2, 16), (8, 3, 3), (8, 2, 16), (1, 2, 16), (16, 2, 4), (8, 1, 16), (3, 5, 9)]
    for maximum, n_min, n_max in params:
        for _ in range(60):
            n = rng.choice([0, 1, 2, 3, 4, 5, 8, 13, 32, 64, 200])
            alphabet = rng.choice([2, 3, 5, 40])
            hist = [rng.randrange(alphabet) for _ in range(n)]
            if n > 6 and rng.random() < 0.5:  # plant a repeat of the suffix
                size = rng.randint(1, min(n // 2, 18))
                at = rng.randrange(0, n - size)
                hist[at:at + size] = hist[n - size:]
            draft_cases.append({"history": hist, "maximum": maximum, "n_min": n_min, "n_max": n_max,
                                "draft": audit.draft(hist, maximum, n_min, n_max)})
    replay_cases = []
    for maximum, n_min, n_max in [(4, 2, 16), (8, 3, 3), (2, 2, 16)]:
        for _ in range(20):
            n = rng.choice([1, 5, 30, 120])
            alphabet = rng.choice([2, 4, 50])
            toks = [rng.randrange(alphabet) for _ in range(n)] + [999]
            r = audit.replay(toks, 999, maximum, n_min, n_max)
            replay_cases.append({"tokens": toks, "eos": 999, "maximum": maximum, "n_min": n_min,
                                 "n_max": n_max, "calls": r["oracleReplayTargetCalls"],
                                 "drafted_calls": r["callsWithDraft"], "proposed": r["proposedTokens"],
                                 "accepted": r["acceptedDraftTokens"], "input_work": r["targetInputTokenWork"]})
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "ngram_draft.json"), "w") as f:
        json.dump({"source": "cpu-lab/moss_ngram_audit.py:16 draft()", "cases": draft_cases}, f)
    with open(os.path.join(here, "ngram_replay.json"), "w") as f:
        json.dump({"source": "cpu-lab/moss_ngram_audit.py:28 replay()", "cases": replay_cases}, f)
    print(len(draft_cases), len(replay_cases))


if __name__ == "__main__":
    main()
