"""Strategy evaluation of the swarm side mode: RSI mean-reversion variants scored on daily closes,
with Monte-Carlo Sharpe confidence intervals.

Semantics follow the reference's swarm page (swarm.html):

* ``rsi``: Wilder's RSI, the first ``period`` outputs 50, the seed average over the first ``period``
  changes, then the (period-1)/period recursive smoothing; 100 when the average loss is 0 (:125-141);
* ``strategy_returns``: from bar 2 on, a position sized by how far the previous bar's RSI is past the
  long/short threshold (capped at 1, scaled by ``short - 50``), optionally confirmed by the previous
  bar's return sign, applied to the equal-weight return of the universe (:179-211);
* ``sharpe`` / ``full_metrics``: on the returns shifted by one bar (a leading 0, the last dropped):
  annualised Sharpe (-9 when flat or shorter than 10 bars), Calmar, max drawdown, win rate, total
  return (:143-177), rounded like the reference;
* ``monte_carlo_sharpe``: GBM paths with the strategy's annualised drift and volatility, each scored
  by ``sharpe``; the 5% / 95% order statistics give the interval (:214-268). The paths run on the GPU
  (``_C.mc_sharpe``, one thread per path) or, without a GPU, in numpy.
"""
from __future__ import annotations

import math
from typing import Sequence

import numpy as np

ANNUAL = 252
MC_PATHS = 50_000
MC_STEPS = 252


def rsi(prices: Sequence[float], period: int) -> np.ndarray:
    p = np.asarray(prices, dtype=np.float64)
    out = np.empty(len(p))
    ch = np.diff(p)
    gain = np.where(ch[:period] > 0, ch[:period], 0.0).sum() / period
    loss = np.where(ch[:period] < 0, -ch[:period], 0.0).sum() / period
    out[:period] = 50.0
    out[period] = 100.0 if loss == 0 else 100.0 - 100.0 / (1.0 + gain / loss)
    for i in range(period + 1, len(p)):
        c = ch[i - 1]
        gain = (gain * (period - 1) + (c if c > 0 else 0.0)) / period
        loss = (loss * (period - 1) + (-c if c < 0 else 0.0)) / period
        out[i] = 100.0 if loss == 0 else 100.0 - 100.0 / (1.0 + gain / loss)
    return out


def strategy_returns(params: dict, data: dict) -> np.ndarray:
    sig = np.asarray(data[params["signalTicker"]], dtype=np.float64)
    period = params.get("rsiPeriod") or 14
    long_t = params.get("longThreshold") or 38
    short_t = params.get("shortThreshold") or 62
    denom = short_t - 50
    universe = params.get("universe") or ["SPY"]
    momentum = bool(params.get("momentumConfirm", False))
    r = rsi(sig, period)
    closes = [np.asarray(data[t], dtype=np.float64) for t in universe]
    out = []
    for i in range(2, len(sig)):
        rv = r[i - 1]
        prev = (sig[i - 1] - sig[i - 2]) / sig[i - 2]
        pos = 0.0
        if momentum:
            if rv < long_t and prev < 0:
                pos = min((long_t - rv) / denom, 1.0)
            elif rv > short_t and prev > 0:
                pos = -min((rv - short_t) / denom, 1.0)
        else:
            if rv < long_t:
                pos = min((long_t - rv) / denom, 1.0)
            elif rv > short_t:
                pos = -min((rv - short_t) / denom, 1.0)
        ret = 0.0
        if pos != 0:
            ret = sum((c[i] - c[i - 1]) / c[i - 1] for c in closes) / len(closes) * pos
        out.append(ret)
    return np.asarray(out)


def _shifted(returns: np.ndarray) -> np.ndarray:
    r = np.asarray(returns, dtype=np.float64)
    return np.concatenate([[0.0], r[:-1]]) if len(r) else np.zeros(1)


def sharpe(returns) -> float:
    r = np.asarray(returns, dtype=np.float64)
    if len(r) < 10:
        return -9.0
    x = _shifted(r)
    m = x.mean()
    s = math.sqrt(((x - m) ** 2).mean())
    return m / s * math.sqrt(ANNUAL) if s > 1e-9 else -9.0


def full_metrics(returns) -> dict:
    x = _shifted(np.asarray(returns, dtype=np.float64))
    n = len(x)
    m = x.mean()
    s = math.sqrt(((x - m) ** 2).mean())
    sh = m / s * math.sqrt(ANNUAL) if s > 1e-9 else -9.0
    cum = np.cumprod(1.0 + x)
    peak = np.maximum(np.maximum.accumulate(cum), 1.0)
    max_dd = float(min(((cum - peak) / peak).min(), 0.0))
    wins = int((x > 0).sum())
    calmar = (m * ANNUAL) / abs(max_dd) if abs(max_dd) > 1e-9 else -9.0
    return {
        "sharpe": round(sh, 6),
        "calmar": round(calmar, 6),
        "max_drawdown": round(max_dd, 6),
        "win_rate": round(wins / n, 4),
        "total_return": round(float(cum[-1]) - 1.0, 4),
    }


def gbm_moments(base_returns) -> tuple[float, float]:
    r = np.asarray(base_returns, dtype=np.float64)
    mu = r.mean() * ANNUAL
    sigma = math.sqrt(((r - r.mean()) ** 2).mean() * ANNUAL)
    return mu, sigma


def mc_sharpes_numpy(mu: float, sigma: float, n_paths: int, steps: int = MC_STEPS, seed: int = 0,
                     chunk: int = 8192) -> np.ndarray:
    """CPU restatement of the Monte-Carlo (vectorised over paths)."""
    rng = np.random.default_rng(seed)
    dt = 1.0 / ANNUAL
    drift = (mu - 0.5 * sigma * sigma) * dt
    diff = sigma * math.sqrt(dt)
    out = np.empty(n_paths)
    for s0 in range(0, n_paths, chunk):
        k = min(chunk, n_paths - s0)
        r = np.expm1(drift + diff * rng.standard_normal((k, steps - 1)))
        x = np.concatenate([np.zeros((k, 1)), r[:, :-1]], axis=1)
        m = x.mean(axis=1)
        sd = np.sqrt(((x - m[:, None]) ** 2).mean(axis=1))
        out[s0:s0 + k] = np.where(sd > 1e-9, m / np.maximum(sd, 1e-300) * math.sqrt(ANNUAL), -9.0)
    return out


def mc_sharpes(mu: float, sigma: float, n_paths: int = MC_PATHS, steps: int = MC_STEPS, seed: int = 0,
               device=None) -> np.ndarray:
    import torch
    if device is not None and torch.device(device).type == "cuda":
        from ..ops._ext import ext
        d = torch.device(device).index or 0
        return ext().mc_sharpe(n_paths, steps, mu, sigma, float(ANNUAL), seed, d).double().cpu().numpy()
    return mc_sharpes_numpy(mu, sigma, n_paths, steps, seed)


def run_variant(variant: dict, data: dict, n_paths: int = MC_PATHS, seed: int = 0, device=None) -> dict:
    """One variant: base metrics on the data, then the Monte-Carlo interval (swarm.html:238-274)."""
    base = strategy_returns(variant, data)
    metrics = full_metrics(base)
    mu, sigma = gbm_moments(base)
    sh = np.sort(mc_sharpes(mu, sigma, n_paths, MC_STEPS, seed + int(variant.get("id", 0)), device))
    mean = float(sh.mean())
    metrics.update({
        "sharpe_ci_low": round(float(sh[int(n_paths * 0.05)]), 6),
        "sharpe_ci_high": round(float(sh[int(n_paths * 0.95)]), 6),
        "mc_mean_sharpe": round(mean, 6),
        "mc_std_sharpe": round(float(math.sqrt(((sh - mean) ** 2).mean())), 6),
    })
    return {"params": variant, "metrics": metrics}


def variant_grid() -> list[dict]:
    """The reference's variant grid (scripts/prepare_swarm.ts:96-120): 1,120 RSI variants."""
    variants = []
    i = 0
    universes = [["SPY"], ["SPY", "QQQ"], ["SPY", "QQQ", "IWM"], ["SPY", "IWM"], ["QQQ", "IWM"]]
    for ticker in ["SPY", "QQQ", "IWM"]:
        for period in [7, 10, 12, 14, 18, 21, 28]:
            for lo, hi in [(25, 75), (30, 70), (33, 67), (35, 65), (38, 62), (40, 60), (42, 58), (45, 55)]:
                for uni in universes:
                    for mom in (False, True):
                        if ticker not in uni:
                            continue
                        variants.append({
                            "id": i, "signalTicker": ticker, "rsiPeriod": period, "longThreshold": lo,
                            "shortThreshold": hi, "universe": uni, "momentumConfirm": mom,
                            "description": f"{ticker} RSI({period}) {lo}/{hi} {'+mom' if mom else ''} -> {'+'.join(uni)}",
                        })
                        i += 1
    return variants


def synthetic_market(tickers=("SPY", "QQQ", "GLD", "TLT", "IWM"), bars: int = 504, seed: int = 0) -> dict:
    """Seeded correlated GBM closes standing in for the downloaded daily bars (no network here)."""
    rng = np.random.default_rng(seed)
    k = len(tickers)
    corr = np.full((k, k), 0.5) + 0.5 * np.eye(k)
    chol = np.linalg.cholesky(corr)
    z = rng.standard_normal((bars, k)) @ chol.T
    vol = np.linspace(0.15, 0.30, k) / math.sqrt(ANNUAL)
    drift = 0.07 / ANNUAL - 0.5 * vol ** 2
    logp = np.log(100.0) + np.cumsum(drift + vol * z, axis=0)
    return {t: np.exp(logp[:, j]).tolist() for j, t in enumerate(tickers)}
