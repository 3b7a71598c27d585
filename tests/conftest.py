from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {key: data[key] for key in data.files}


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle

    oracle.build()
    return oracle


def first_difference(a, b) -> int:
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))


def penalised_scores(logits: np.ndarray, seen, penalty: float) -> np.ndarray:
    """The reference sampler's scores at temperature 1 (decoder.py:324-333): a seen token's logit is
    divided by the penalty when positive and multiplied by it otherwise (float32)."""
    s = np.asarray(logits, np.float32).copy()
    if penalty != 1.0:
        inv = np.float32(1.0 / penalty)
        for t in set(int(x) for x in seen):
            s[t] = s[t] * (inv if s[t] > 0 else np.float32(penalty))
    return s


def check_greedy_stream(ours, stream, prefill_logits, step_logits, penalty: float, tol: float) -> int:
    """`ours` equals the reference's (penalised) greedy `stream` token for token, or the two part at a
    step where the reference's own choice had a runner-up within `tol` of it (a near-tie that logits
    inside the parity tolerance may resolve either way; tol = twice that tolerance). step_logits[i] are
    the reference logits that chose stream[i + 1], prefill_logits chose stream[0]. Returns the number
    of leading tokens that agree."""
    ours, stream = [int(x) for x in ours], [int(x) for x in stream]
    d = first_difference(ours, stream)
    if d < min(len(ours), len(stream)):
        logits = prefill_logits if d == 0 else step_logits[d - 1]
        s = penalised_scores(logits, stream[:d], penalty)
        gap = float(s[stream[d]] - s[ours[d]])
        assert 0.0 <= gap < tol, f"streams part at token {d} where the reference's margin is {gap:.4f} (>= {tol})"
    return d
