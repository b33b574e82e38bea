"""Seeded synthetic inputs standing in for the reference's private teacher data.

The reference trains on PSV/HCPE teacher files (docs/spec/10-cuda-oxide-tickets.md:503-521)
that are not available; these generators reproduce their shapes, index ranges
and value distributions:

* HalfKP (125388 = 81 kings x 1548 piece-squares): per perspective a king
  k ~ U{0..80} and 38 distinct piece ids p ~ U[0,1548); feature = k*1548 + p
  (crates/bulletou_lib/src/game/inputs/shogi_halfkp.rs:26-40);
* KPPT: 38 distinct BonaPieces per view; KPP = all 703 pairs a<b,
  k*1548^2 + a*1548 + b (shogi_kpp.rs:14); KKP = k*81*1548 + k'*1548 + p;
  KK = k*81 + k';
* HalfKA_hm2 (73305 = 45 mirrored king buckets x 1629): per perspective a
  king bucket k ~ U{0..44} and 40 distinct pieces p ~ U[0,1629); feature =
  k*1629 + p (shogi_halfka_hm2.rs:106-260); LayerStack bucket ~ U{0..8}
  (k3k3) or Zipf(1.1) over 81 buckets through a seeded permutation (k9k9);
* weights ~ N(0, 0.01); targets t = 0.5*r + 0.5*sigmoid(score/600) with
  score = round(N(0,600)) clipped to +-3000 and r in {0, 1/2, 1}
  (teacher_batch.rs:1709-1746 blend with lambda = 0.5); entry weight 1.

numpy's PCG64 generator, one stream per (seed, rank).
"""
from __future__ import annotations

import numpy as np

HALFKP_KINGS = 81
HALFKP_PIECES = 1548
HALFKP_INPUTS = HALFKP_KINGS * HALFKP_PIECES  # 125388
HALFKP_ACTIVE = 38
KPP_INPUTS = HALFKP_KINGS * HALFKP_PIECES * HALFKP_PIECES  # 194100624
KKP_INPUTS = HALFKP_KINGS * HALFKP_KINGS * HALFKP_PIECES  # 10156428
KK_INPUTS = HALFKP_KINGS * HALFKP_KINGS  # 6561
KPP_PAIRS = HALFKP_ACTIVE * (HALFKP_ACTIVE - 1) // 2  # 703


def rng_for(seed: int, rank: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, rank]))


def distinct_pieces(rng: np.random.Generator, rows: int, k: int = HALFKP_ACTIVE, n: int = HALFKP_PIECES,
                    sort: bool = False) -> np.ndarray:
    """rows x k distinct values in [0, n)."""
    out = np.empty((rows, k), np.int32)
    chunk = 2048
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        keys = rng.random((r1 - r0, n), dtype=np.float32)
        pick = np.argpartition(keys, k, axis=1)[:, :k]
        out[r0:r1] = pick
    if sort:
        out.sort(axis=1)
    return out


def halfkp_indices(rng: np.random.Generator, batch: int) -> tuple[np.ndarray, np.ndarray]:
    """(stm, nstm) int32 [batch*38], perspectives drawn independently."""
    views = []
    for _ in range(2):
        kings = rng.integers(0, HALFKP_KINGS, size=(batch, 1), dtype=np.int32)
        pieces = distinct_pieces(rng, batch)
        views.append((kings * HALFKP_PIECES + pieces).astype(np.int32).reshape(-1))
    return views[0], views[1]


def targets(rng: np.random.Generator, batch: int, scale: float = 600.0, lam: float = 0.5) -> tuple[np.ndarray, np.ndarray]:
    """(targets, entry_weights) float32 [batch]."""
    score = np.clip(np.rint(rng.normal(0.0, 600.0, size=batch)), -3000, 3000).astype(np.float32)
    result = rng.integers(-1, 2, size=batch).astype(np.float32)
    r = (result + 1.0) * 0.5
    t = (1.0 - lam) * r + lam * (1.0 / (1.0 + np.exp(-score / scale)))
    return t.astype(np.float32), np.ones(batch, np.float32)


def halfkp_weights(rng: np.random.Generator, input_size: int = HALFKP_INPUTS, l1: int = 256, l2: int = 32,
                   l3: int = 32, std: float = 0.01) -> dict:
    shapes = {"l0w": input_size * l1, "l0b": l1, "l1w": 2 * l1 * l2, "l1b": l2, "l2w": l2 * l3, "l2b": l3,
              "outw": l3, "outb": 1}
    return {k: rng.normal(0.0, std, size=n).astype(np.float32) for k, n in shapes.items()}


def halfkp_batch(seed: int, batch: int, rank: int = 0) -> dict:
    rng = rng_for(seed, rank)
    stm, nstm = halfkp_indices(rng, batch)
    t, w = targets(rng, batch)
    return {"stm": stm, "nstm": nstm, "targets": t, "entry_weights": w, "batch": batch, "max_active": HALFKP_ACTIVE}


def kppt_indices(rng: np.random.Generator, batch: int, component: str) -> tuple[np.ndarray, np.ndarray, int, int]:
    """(stm, nstm, input_size, max_active) for component 'kk' | 'kkp' | 'kpp'."""
    views = []
    if component == "kpp":
        iu, ju = np.triu_indices(HALFKP_ACTIVE, k=1)
        for _ in range(2):
            k = rng.integers(0, HALFKP_KINGS, size=(batch, 1)).astype(np.int64)
            p = distinct_pieces(rng, batch, sort=True).astype(np.int64)
            idx = k * HALFKP_PIECES * HALFKP_PIECES + p[:, iu] * HALFKP_PIECES + p[:, ju]
            views.append(idx.astype(np.int32).reshape(-1))
        return views[0], views[1], KPP_INPUTS, KPP_PAIRS
    if component == "kkp":
        for _ in range(2):
            k0 = rng.integers(0, HALFKP_KINGS, size=(batch, 1)).astype(np.int64)
            k1 = rng.integers(0, HALFKP_KINGS, size=(batch, 1)).astype(np.int64)
            p = distinct_pieces(rng, batch).astype(np.int64)
            views.append((k0 * HALFKP_KINGS * HALFKP_PIECES + k1 * HALFKP_PIECES + p).astype(np.int32).reshape(-1))
        return views[0], views[1], KKP_INPUTS, HALFKP_ACTIVE
    if component == "kk":
        for _ in range(2):
            k0 = rng.integers(0, HALFKP_KINGS, size=batch)
            k1 = rng.integers(0, HALFKP_KINGS, size=batch)
            views.append((k0 * HALFKP_KINGS + k1).astype(np.int32))
        return views[0], views[1], KK_INPUTS, 1
    raise ValueError(f"unknown KPPT component {component!r}")


HM2_KINGS = 45
HM2_PIECES = 1629
HM2_INPUTS = HM2_KINGS * HM2_PIECES  # 73305
HM2_ACTIVE = 40


def hm2_indices(rng: np.random.Generator, batch: int) -> tuple[np.ndarray, np.ndarray]:
    """(stm, nstm) int32 [batch*40] HalfKA_hm2 features, perspectives independent."""
    views = []
    for _ in range(2):
        kings = rng.integers(0, HM2_KINGS, size=(batch, 1), dtype=np.int32)
        pieces = distinct_pieces(rng, batch, HM2_ACTIVE, HM2_PIECES)
        views.append((kings * HM2_PIECES + pieces).astype(np.int32).reshape(-1))
    return views[0], views[1]


def layerstack_buckets(rng: np.random.Generator, batch: int, stacks: int = 9, zipf: float = 0.0) -> np.ndarray:
    """Uniform buckets, or Zipf(s) ranks mapped through a seeded permutation."""
    if zipf <= 0.0:
        return rng.integers(0, stacks, size=batch).astype(np.int32)
    ranks = np.arange(1, stacks + 1, dtype=np.float64)
    p = ranks ** -zipf
    p /= p.sum()
    perm = rng.permutation(stacks)
    return perm[rng.choice(stacks, size=batch, p=p)].astype(np.int32)


def sfnn_batch(seed: int, batch: int, rank: int = 0, stacks: int = 9, zipf: float = 0.0) -> dict:
    rng = rng_for(seed, rank)
    stm, nstm = hm2_indices(rng, batch)
    buckets = layerstack_buckets(rng, batch, stacks, zipf)
    t, w = targets(rng, batch)
    return {"stm": stm, "nstm": nstm, "buckets": buckets, "targets": t, "entry_weights": w, "batch": batch,
            "max_active": HM2_ACTIVE}


def sfnn_weights(rng: np.random.Generator, input_size: int = HM2_INPUTS + HM2_PIECES, ft: int = 1536,
                 l1_hidden: int = 15, l1_skip: bool = True, l2: int = 32, stacks: int = 9, shared_l1: bool = True,
                 shared_l2_l3: bool = False, std: float = 0.01) -> dict:
    """N(0, std) weights of an SFNN LayerStack net (absent shared factors are None)."""
    o = l1_hidden + int(l1_skip)
    i2 = 2 * l1_hidden
    shapes = {"l0w": input_size * ft, "l0b": ft, "l1w": stacks * o * ft, "l1b": stacks * o,
              "l2w": stacks * l2 * i2, "l2b": stacks * l2, "l3w": stacks * l2, "l3b": stacks}
    if shared_l1:
        shapes.update({"l1fw": ft * o, "l1fb": o})
    if shared_l2_l3:
        shapes.update({"l2fw": l2 * i2, "l2fb": l2, "l3fw": l2, "l3fb": 1})
    out = {k: rng.normal(0.0, std, size=n).astype(np.float32) for k, n in shapes.items()}
    for k in ("l1fw", "l1fb", "l2fw", "l2fb", "l3fw", "l3fb"):
        out.setdefault(k, None)
    return out
