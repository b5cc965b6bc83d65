"""
search.py — search strategies that choose which variants get compiled and timed.

Same interface as the reference (src/search.py:52-78): `suggest(n)`,
`update(params, ms)`, `best()`, plus `make_strategy` (:395-422) and
`ConvergenceLogger` (:427-461). Differences:

  * the strategy drives the sweep: the tuner evaluates only what `suggest`
    returns (the reference submitted every enumerated variant and only fed
    results back, autotune.py:301-317);
  * `BayesianOptStrategy` is a self-contained Gaussian-process / expected-
    improvement search over the finite grid (scikit-optimize is not
    installed here; the reference fell back to a grid): each parameter is
    encoded on [0, 1] (log2 for powers of two, rank for categories), an RBF
    GP is fit to standardised log-latencies, and the unevaluated point with
    the largest expected improvement is proposed next (Snoek et al., 2012);
  * `SuccessiveHalvingStrategy` gives each round a sample budget
    (`budget()`), r_min · eta^round, so early rounds are cheap and survivors
    are re-measured with more samples (Jamieson & Talwalkar, 2016).
"""

from __future__ import annotations

import itertools
import json
import math
import random
from abc import ABC, abstractmethod
from pathlib import Path
from typing import List, Optional, Sequence

import numpy as np

from parser import is_valid


def _param_keys(space: dict) -> list[str]:
    return [k for k in space if not k.startswith("_")]


def expand_space(space: dict, kernel: str = "") -> List[dict]:
    """Valid points of a search space, in grid order."""
    keys = _param_keys(space)
    out = []
    for combo in itertools.product(*(space[k] for k in keys)):
        p = dict(zip(keys, combo))
        if not kernel or is_valid(kernel, p):
            out.append(p)
    return out


def _key(params: dict) -> str:
    return "_".join(f"{k}{v}" for k, v in sorted(params.items()))


class SearchStrategy(ABC):
    """suggest / update / best."""

    @abstractmethod
    def suggest(self, n: int = 1) -> List[dict]:
        """Up to n configurations to evaluate next ([] when the strategy is done)."""

    @abstractmethod
    def update(self, params: dict, result_ms: float) -> None:
        """Record the measured latency of params (inf for a failed variant)."""

    @abstractmethod
    def best(self) -> Optional[dict]:
        """Params with the lowest latency so far."""

    def budget(self) -> Optional[int]:
        """Timing samples the next suggested batch should get (None: caller's default)."""
        return None

    @property
    def name(self) -> str:
        return self.__class__.__name__


class GridSearchStrategy(SearchStrategy):
    """Exhaustive traversal of every valid point."""

    def __init__(self, space: dict, kernel: str = "") -> None:
        self._queue = expand_space(space, kernel)
        self._ptr = 0
        self._results: list[tuple[dict, float]] = []

    def suggest(self, n: int = 1) -> List[dict]:
        batch = self._queue[self._ptr:self._ptr + n]
        self._ptr += len(batch)
        return batch

    def update(self, params: dict, result_ms: float) -> None:
        self._results.append((params, result_ms))

    def best(self) -> Optional[dict]:
        ok = [r for r in self._results if math.isfinite(r[1])]
        return min(ok, key=lambda r: r[1])[0] if ok else None

    @property
    def total(self) -> int:
        return len(self._queue)

    @property
    def remaining(self) -> int:
        return max(0, len(self._queue) - self._ptr)


def _encode(space: dict, points: List[dict]) -> np.ndarray:
    """Map each parameter to [0, 1]: log2 scale for positive numbers, rank otherwise."""
    keys = _param_keys(space)
    cols = []
    for k in keys:
        vals = list(space[k])
        numeric = all(isinstance(v, (int, float)) and not isinstance(v, bool) and v > 0 for v in vals)
        if numeric and len(vals) > 1:
            lv = np.log2(np.array(vals, dtype=np.float64))
            lo, hi = lv.min(), lv.max()
            col = [(math.log2(p[k]) - lo) / (hi - lo) if hi > lo else 0.0 for p in points]
        else:
            idx = {repr(v): i for i, v in enumerate(vals)}
            den = max(1, len(vals) - 1)
            col = [idx[repr(p[k])] / den for p in points]
        cols.append(col)
    return np.array(cols, dtype=np.float64).T if cols else np.zeros((len(points), 0))


class BayesianOptStrategy(SearchStrategy):
    """
    GP-EI over the finite grid. The first `n_initial` points are a seeded
    random design; afterwards every suggestion maximises expected improvement
    of log-latency under an RBF Gaussian process. At most `n_calls` points
    are suggested.
    """

    def __init__(self, space: dict, kernel: str = "", n_calls: int = 40, n_initial: Optional[int] = None,
                 length_scale: float = 0.35, noise: float = 1e-3, seed: int = 0, anchors: Sequence[dict] = ()) -> None:
        self._space = space
        self._cands = expand_space(space, kernel)
        self._X = _encode(space, self._cands)
        self._n_calls = min(n_calls, len(self._cands))
        self._n_initial = n_initial if n_initial is not None else min(10, max(2, self._n_calls // 4))
        self._ls = length_scale
        self._noise = noise
        self._rng = random.Random(seed)
        self._suggested: set[int] = set()
        self._obs: dict[int, float] = {}
        self._results: list[tuple[dict, float]] = []
        self._index = {_key(p): i for i, p in enumerate(self._cands)}
        # anchor points (e.g. the default configuration) open the initial design
        self._anchors = [self._index[_key(p)] for p in anchors if _key(p) in self._index]

    def _kernel(self, A: np.ndarray, B: np.ndarray) -> np.ndarray:
        d2 = ((A[:, None, :] - B[None, :, :]) ** 2).sum(-1)
        return np.exp(-0.5 * d2 / (self._ls ** 2))

    def _posterior(self, idx_obs: list[int], y: np.ndarray, idx_q: list[int]) -> tuple[np.ndarray, np.ndarray]:
        Xo, Xq = self._X[idx_obs], self._X[idx_q]
        K = self._kernel(Xo, Xo) + self._noise * np.eye(len(idx_obs))
        L = np.linalg.cholesky(K)
        alpha = np.linalg.solve(L.T, np.linalg.solve(L, y))
        Ks = self._kernel(Xq, Xo)
        mu = Ks @ alpha
        v = np.linalg.solve(L, Ks.T)
        var = np.clip(1.0 - (v ** 2).sum(0), 1e-12, None)
        return mu, np.sqrt(var)

    def expected_improvement(self) -> dict[int, float]:
        """EI of every unevaluated candidate (exposed for tests and logging)."""
        from scipy.stats import norm
        obs = [i for i in self._obs if math.isfinite(self._obs[i])]
        free = [i for i in range(len(self._cands)) if i not in self._suggested]
        if not obs or not free:
            return {}
        y = np.log(np.array([self._obs[i] for i in obs]))
        mu_y, sd_y = y.mean(), y.std() or 1.0
        yn = (y - mu_y) / sd_y
        mu, sd = self._posterior(obs, yn, free)
        best = yn.min()
        z = (best - mu) / sd
        ei = (best - mu) * norm.cdf(z) + sd * norm.pdf(z)
        return dict(zip(free, ei.tolist()))

    def suggest(self, n: int = 1) -> List[dict]:
        out: List[dict] = []
        while len(out) < n and len(self._suggested) < self._n_calls:
            free = [i for i in range(len(self._cands)) if i not in self._suggested]
            if not free:
                break
            pending = [a for a in self._anchors if a not in self._suggested]
            if pending:
                i = pending[0]
            elif len(self._obs) < self._n_initial or len(self._suggested) < self._n_initial:
                i = self._rng.choice(free)
            else:
                ei = self.expected_improvement()
                i = max(ei, key=ei.get) if ei else self._rng.choice(free)
            self._suggested.add(i)
            out.append(self._cands[i])
            if len(self._obs) >= self._n_initial:
                break  # one model-based point per refit
        return out

    def update(self, params: dict, result_ms: float) -> None:
        i = self._index.get(_key(params))
        self._results.append((params, result_ms))
        if i is not None:
            self._suggested.add(i)
            # a failed variant is treated as a very slow one so the GP avoids its region
            worst = max([v for v in self._obs.values() if math.isfinite(v)] or [1.0])
            self._obs[i] = result_ms if math.isfinite(result_ms) else 10.0 * worst

    def best(self) -> Optional[dict]:
        ok = [r for r in self._results if math.isfinite(r[1])]
        return min(ok, key=lambda r: r[1])[0] if ok else None


class SuccessiveHalvingStrategy(SearchStrategy):
    """
    Successive halving: n_configs random points, each round timed with
    r_min·eta^round samples; the best 1/eta survive to the next round.
    """

    def __init__(self, space: dict, kernel: str = "", n_configs: int = 80, eta: int = 2, r_min: int = 5,
                 seed: int = 0, anchors: Sequence[dict] = ()) -> None:
        cands = expand_space(space, kernel)
        rng = random.Random(seed)
        rng.shuffle(cands)
        # anchor points (e.g. the default configuration) always enter the first round
        keys = {_key(p) for p in cands}
        first = [p for p in anchors if _key(p) in keys]
        first_keys = {_key(p) for p in first}
        cands = first + [p for p in cands if _key(p) not in first_keys]
        self._bracket = cands[:min(n_configs, len(cands))]
        self._eta = eta
        self._r_min = r_min
        self._ptr = 0
        self._round = 0
        self._round_results: dict[str, float] = {}
        self._best: dict[str, tuple[dict, float]] = {}
        self._done = False

    def budget(self) -> Optional[int]:
        return self._r_min * (self._eta ** self._round)

    def suggest(self, n: int = 1) -> List[dict]:
        if self._done:
            return []
        batch = self._bracket[self._ptr:self._ptr + n]
        self._ptr += len(batch)
        return batch

    def update(self, params: dict, result_ms: float) -> None:
        k = _key(params)
        self._round_results[k] = result_ms
        if math.isfinite(result_ms) and (k not in self._best or result_ms < self._best[k][1]):
            self._best[k] = (params, result_ms)
        if self._ptr >= len(self._bracket) and all(_key(p) in self._round_results for p in self._bracket):
            self._advance_round()

    def _advance_round(self) -> None:
        ranked = sorted(self._bracket, key=lambda p: self._round_results.get(_key(p), math.inf))
        ranked = [p for p in ranked if math.isfinite(self._round_results.get(_key(p), math.inf))]
        if len(ranked) <= 1:
            self._done = True
            self._bracket = ranked
            return
        self._bracket = ranked[:max(1, len(ranked) // self._eta)]
        self._ptr = 0
        self._round += 1
        self._round_results = {}

    def best(self) -> Optional[dict]:
        if not self._best:
            return None
        return min(self._best.values(), key=lambda x: x[1])[0]

    @property
    def bracket_size(self) -> int:
        return len(self._bracket)

    @property
    def current_round(self) -> int:
        return self._round


def make_strategy(name: str, space: dict, kernel: str = "", n_calls: int = 40, n_configs: int = 80,
                  seed: int = 0, anchors: Sequence[dict] = ()) -> SearchStrategy:
    """'grid' | 'bayesian' | 'sha' (aliases as in the reference). `anchors`:
    points the sampling strategies evaluate first (the grid visits every point)."""
    name = name.lower()
    if name in ("grid", "gridsearch"):
        return GridSearchStrategy(space, kernel)
    if name in ("bayesian", "bayes", "bo"):
        return BayesianOptStrategy(space, kernel, n_calls=n_calls, seed=seed, anchors=anchors)
    if name in ("sha", "successive_halving", "halving"):
        return SuccessiveHalvingStrategy(space, kernel, n_configs=n_configs, seed=seed, anchors=anchors)
    raise ValueError(f"Unknown strategy {name!r}. Choose: grid | bayesian | sha")


class ConvergenceLogger:
    """eval number -> best-so-far latency; saved to results/{kernel}_convergence.json."""

    def __init__(self, kernel: str, results_dir: Path) -> None:
        self._kernel = kernel
        self._path = Path(results_dir) / f"{kernel}_convergence.json"
        self._curve: List[dict] = []
        self._best_ms = float("inf")
        self._eval = 0

    def record(self, params: dict, ms: float) -> None:
        self._eval += 1
        if ms < self._best_ms:
            self._best_ms = ms
        self._curve.append({"eval": self._eval, "ms": ms, "best_ms": self._best_ms, "params": params})

    def save(self) -> None:
        self._path.parent.mkdir(parents=True, exist_ok=True)
        self._path.write_text(json.dumps({"kernel": self._kernel, "n_evals": self._eval,
                                          "best_ms": self._best_ms, "curve": self._curve}, indent=2))
