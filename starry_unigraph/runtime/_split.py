"""Train/val/test split helpers (reference runtime/_split.py:6-44).

Counts are floor(total * ratio); the remainder goes to the splits with the
largest fractional parts; every positive split gets at least one item (taken
from the largest split) when total allows.
"""
from __future__ import annotations


def normalize_split_ratio(split_ratio: dict[str, float] | None) -> dict[str, float]:
    ratio = dict(split_ratio or {})
    train = max(0.0, float(ratio.get("train", 0.7)))
    val = max(0.0, float(ratio.get("val", 0.15)))
    test = max(0.0, float(ratio.get("test", 0.15)))
    total = train + val + test
    if total <= 0:
        return {"train": 0.7, "val": 0.15, "test": 0.15}
    return {"train": train / total, "val": val / total, "test": test / total}


def split_counts(total: int, split_ratio: dict[str, float]) -> dict[str, int]:
    keys = ("train", "val", "test")
    raw = {k: total * split_ratio[k] for k in keys}
    counts = {k: int(raw[k]) for k in keys}
    remainder = total - sum(counts.values())
    if remainder > 0:
        order = sorted(keys, key=lambda k: raw[k] - counts[k], reverse=True)
        for i in range(remainder):
            counts[order[i % len(order)]] += 1
    positive = [k for k in keys if split_ratio[k] > 0]
    if total >= len(positive):
        for k in positive:
            if counts[k] > 0:
                continue
            donor = max(positive, key=lambda item: counts[item])
            if counts[donor] > 1:
                counts[donor] -= 1
                counts[k] += 1
    return counts


def split_bounds(total: int, split: str, split_ratio: dict[str, float]) -> tuple[int, int]:
    if total <= 0:
        return 0, 0
    counts = split_counts(total, split_ratio)
    train_end = min(total, counts["train"])
    val_end = min(total, train_end + counts["val"])
    if split == "train":
        return 0, train_end
    if split == "val":
        return train_end, max(val_end, train_end)
    if split == "test":
        return val_end, total
    raise KeyError(f"Unsupported split: {split!r}")
