"""Strategy swarm on CPU: RSI, metrics and the variant grid against direct restatements, and the chunked
work queue with two worker processes, and the requeue of a departed worker's variants."""
import math

import numpy as np

from bitresearch_b200.swarm import SwarmQueue, full_metrics, rsi, run_swarm, sharpe, strategy_returns, variant_grid
from bitresearch_b200.swarm.strategy import mc_sharpes_numpy, synthetic_market


def test_rsi_matches_wilder_definition():
    p = [44.3, 44.1, 44.2, 43.6, 44.3, 44.8, 45.1, 45.4, 45.8, 46.1, 45.9, 46.0, 45.6, 46.3, 46.3, 46.0, 46.4, 46.2]
    out = rsi(p, 14)
    assert (out[:14] == 50).all()
    ch = np.diff(p)
    g = ch[:14].clip(min=0).mean()
    l = (-ch[:14]).clip(min=0).mean()
    assert math.isclose(out[14], 100 - 100 / (1 + g / l), rel_tol=1e-12)
    g = (g * 13 + max(ch[14], 0)) / 14
    l = (l * 13 + max(-ch[14], 0)) / 14
    assert math.isclose(out[15], 100 - 100 / (1 + g / l), rel_tol=1e-12)
    assert rsi([1, 2, 3, 4, 5, 6], 3)[3] == 100.0  # no losses


def test_metrics_on_shifted_returns():
    r = np.array([0.01, -0.02, 0.03, 0.0, 0.01, -0.01, 0.02, 0.01, -0.005, 0.004, 0.5])  # last one is dropped
    x = np.concatenate([[0.0], r[:-1]])
    m, s = x.mean(), x.std()
    assert math.isclose(sharpe(r), m / s * math.sqrt(252), rel_tol=1e-12)
    met = full_metrics(r)
    cum = np.cumprod(1 + x)
    assert math.isclose(met["total_return"], round(cum[-1] - 1, 4))
    assert met["win_rate"] == round((x > 0).sum() / len(x), 4)
    assert met["max_drawdown"] < 0
    assert sharpe(r[:9]) == -9  # too short
    assert sharpe(np.zeros(20)) == -9  # flat


def test_variant_grid_and_strategy():
    grid = variant_grid()
    assert len(grid) == 1120 and grid[0]["id"] == 0 and grid[-1]["id"] == 1119
    assert all(v["signalTicker"] in v["universe"] for v in grid)
    data = synthetic_market(bars=300, seed=3)
    r = strategy_returns(grid[0], data)
    assert len(r) == 298 and np.isfinite(r).all()
    assert (np.abs(r) > 0).any()


def test_numpy_monte_carlo_sharpe_distribution():
    # zero drift: the simulated Sharpe ratios centre near 0 with spread about 1 (sqrt(252/251) for iid)
    sh = mc_sharpes_numpy(0.0, 0.2, 20000, seed=1)
    assert abs(sh.mean()) < 0.05 and 0.9 < sh.std() < 1.1


def test_queue_assigns_each_variant_once_and_requeues_lost_work():
    vs = [{"id": i, "description": str(i)} for i in range(12)]
    q = SwarmQueue(vs, chunk_size=5)
    a = q.next_chunk("a")
    b = q.next_chunk("b")
    assert [v["id"] for v in a] == [0, 1, 2, 3, 4] and [v["id"] for v in b] == [5, 6, 7, 8, 9]
    q.record({"params": vs[0], "metrics": {"sharpe": 1.0}})
    assert q.release("a") == 4  # a left with 1..4 unfinished
    c = q.next_chunk("c")
    assert [v["id"] for v in c] == [1, 2, 3, 4]


def test_swarm_runs_all_variants_on_two_workers():
    vs = variant_grid()[:12]
    data = synthetic_market(bars=260, seed=5)
    res = run_swarm(vs, data, workers=2, n_paths=500, log=lambda m: None, timeout_s=300)
    assert sorted(r["params"]["id"] for r in res) == list(range(12))
    sh = [r["metrics"]["sharpe"] for r in res]
    assert sh == sorted(sh, reverse=True)
    for r in res:
        m = r["metrics"]
        assert m["sharpe_ci_low"] <= m["mc_mean_sharpe"] <= m["sharpe_ci_high"]
        assert {r["peerId"] for r in res} <= {"worker-0", "worker-1"}


def test_prepare_splits_csv_bars_and_feeds_the_runner(tmp_path, capsys):
    import json
    from bitresearch_b200.swarm import prepare, runner
    csv_dir = tmp_path / "csv"
    csv_dir.mkdir()
    days = prepare.synthetic_bars("2020-06-01", "2021-12-31")["SPY"]["dates"]
    for t in ("SPY", "QQQ", "IWM"):
        rows = ["Date,Open,Close"] + [f"{d},1,{100 + i * 0.1 + (3 if t == 'QQQ' else 0)}" for i, d in enumerate(days)]
        rows.insert(5, f"{days[3]},1,null")  # a missing bar is skipped
        (csv_dir / f"{t.lower()}.csv").write_text("\n".join(rows) + "\n")
    out = tmp_path / "data"
    assert prepare.main(["--csv-dir", str(csv_dir), "--out", str(out), "--val-end", "2021-12-31"]) == 0
    train = json.loads((out / "train.json").read_text())
    val = json.loads((out / "val.json").read_text())
    assert set(train) == {"SPY", "QQQ", "IWM"}
    assert all(d <= "2020-12-31" for d in train["SPY"]["dates"]) and all(d > "2020-12-31" for d in val["SPY"]["dates"])
    assert len(train["SPY"]["dates"]) + len(val["SPY"]["dates"]) == len(days)
    cfg = json.loads((out / "config.json").read_text())
    assert cfg["chunkSize"] == 5 and len(cfg["variants"]) == 1120
    capsys.readouterr()
    res_path = tmp_path / "res.json"
    assert runner.main(["--variants", str(out / "config.json"), "--data", str(out / "val.json"), "--limit", "3",
                        "--paths", "500", "--workers", "1", "--out", str(res_path)]) == 0
    res = json.loads(res_path.read_text())
    assert len(res) == 3 and all("sharpe_ci_low" in r["metrics"] for r in res)


def test_prepare_without_input_writes_synthetic_business_days(tmp_path):
    import datetime
    import json
    from bitresearch_b200.swarm import prepare
    assert prepare.main(["--out", str(tmp_path)]) == 0
    a = json.loads((tmp_path / "all.json").read_text())
    assert set(a) == set(prepare.TICKERS)
    assert all(datetime.date.fromisoformat(d).weekday() < 5 for d in a["SPY"]["dates"][:50])
