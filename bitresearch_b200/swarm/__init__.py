"""Strategy swarm: a task-parallel side mode (RSI variants scored with Monte-Carlo Sharpe intervals)."""
from .runner import SwarmQueue, run_swarm
from .strategy import full_metrics, mc_sharpes, rsi, run_variant, sharpe, strategy_returns, variant_grid

__all__ = ["SwarmQueue", "run_swarm", "full_metrics", "mc_sharpes", "rsi", "run_variant", "sharpe",
           "strategy_returns", "variant_grid"]
