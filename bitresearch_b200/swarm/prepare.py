"""Data preparation of the strategy swarm: daily closes split into train / validation periods by date,
plus the variant list (the reference's scripts/prepare_swarm.ts, which downloads Yahoo Finance bars
for SPY, QQQ, GLD, TLT, IWM from 2010 and splits at 2020-12-31 / 2022-12-31).

There is no download here: the bars come from local files, either the reference's ``all.json``
(``{ticker: {"dates": [...], "close": [...]}}``) or one CSV per ticker with ``Date`` and ``Close``
(or ``Adj Close``) columns, as exported by most data vendors. Without input, seeded synthetic bars on
business days stand in. The outputs match the reference's: ``all.json``, ``train.json``, ``val.json``
and ``config.json`` (``{"variants": [...], "chunkSize": 5}``).

  python -m bitresearch_b200.swarm.prepare [--input all.json | --csv-dir DIR] [--out public/data]
"""
from __future__ import annotations

import argparse
import csv
import datetime
import json
import os
import sys

from .strategy import synthetic_market, variant_grid

TICKERS = ("SPY", "QQQ", "GLD", "TLT", "IWM")
START, TRAIN_END, VAL_END = "2010-01-01", "2020-12-31", "2022-12-31"


def load_csv_dir(path: str) -> dict:
    """``<TICKER>.csv`` files with a Date column and a Close (or Adj Close) column; empty rows skipped."""
    out = {}
    for name in sorted(os.listdir(path)):
        if not name.lower().endswith(".csv"):
            continue
        dates, close = [], []
        with open(os.path.join(path, name), newline="") as f:
            for row in csv.DictReader(f):
                v = row.get("Close") or row.get("close") or row.get("Adj Close") or ""
                d = row.get("Date") or row.get("date") or ""
                try:
                    c = float(v)
                except ValueError:
                    continue  # "null" / missing bars, as the reference drops them
                if d:
                    dates.append(d[:10])
                    close.append(c)
        out[os.path.splitext(name)[0].upper()] = {"dates": dates, "close": close}
    return out


def synthetic_bars(start: str = START, end: str = VAL_END, seed: int = 0) -> dict:
    """Seeded synthetic closes on business days between ``start`` and ``end``."""
    d0, d1 = datetime.date.fromisoformat(start), datetime.date.fromisoformat(end)
    days = [d0 + datetime.timedelta(k) for k in range((d1 - d0).days + 1)]
    days = [d.isoformat() for d in days if d.weekday() < 5]
    closes = synthetic_market(TICKERS, bars=len(days), seed=seed)
    return {t: {"dates": days, "close": closes[t]} for t in TICKERS}


def split(all_data: dict, train_end: str = TRAIN_END, val_end: str = VAL_END) -> tuple[dict, dict]:
    """Bars up to ``train_end`` train, then up to ``val_end`` validation (ISO dates compare as strings)."""
    train, val = {}, {}
    for t, d in all_data.items():
        tr = {"dates": [], "close": []}
        va = {"dates": [], "close": []}
        for day, c in zip(d["dates"], d["close"]):
            if day <= train_end:
                tr["dates"].append(day)
                tr["close"].append(c)
            elif day <= val_end:
                va["dates"].append(day)
                va["close"].append(c)
        train[t], val[t] = tr, va
    return train, val


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="prepare swarm data: train/val closes and the variant list")
    ap.add_argument("--input", default="", help="all.json in the reference's format")
    ap.add_argument("--csv-dir", default="", help="one <TICKER>.csv per ticker (Date, Close)")
    ap.add_argument("--out", default=os.path.join("public", "data"))
    ap.add_argument("--train-end", default=TRAIN_END)
    ap.add_argument("--val-end", default=VAL_END)
    ap.add_argument("--seed", type=int, default=0, help="synthetic bars when no input is given")
    args = ap.parse_args(argv)
    if args.input:
        with open(args.input) as f:
            all_data = json.load(f)
    elif args.csv_dir:
        all_data = load_csv_dir(args.csv_dir)
    else:
        print("no --input / --csv-dir: writing seeded synthetic bars", file=sys.stderr)
        all_data = synthetic_bars(seed=args.seed)
    train, val = split(all_data, args.train_end, args.val_end)
    os.makedirs(args.out, exist_ok=True)
    for name, obj in (("all.json", all_data), ("train.json", train), ("val.json", val),
                      ("config.json", {"variants": variant_grid(), "chunkSize": 5})):
        with open(os.path.join(args.out, name), "w") as f:
            json.dump(obj, f)
    first = next(iter(train))
    print(f"train bars: {len(train[first]['dates'])}, val bars: {len(val[first]['dates'])}, "
          f"variants: {len(variant_grid())} -> {args.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
