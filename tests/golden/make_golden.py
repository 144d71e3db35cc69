"""Generates the golden fixtures in this directory from an independent
pure-Python restatement of the training semantics (no numpy arithmetic on the
decision path, exact rational arithmetic for fused multiply-add).

    python tests/golden/make_golden.py

The reference's training arithmetic lives in XGBoost 3.4.1, which is not
vendored in the reference repository and not installed here, so these
fixtures pin the C++ oracle and the CUDA path to a second, separately written
statement of the same rules rather than to XGBoost itself.  Inputs are small
seeded synthetic matrices (with NaN, ties and signed zeros).
"""
from __future__ import annotations

import json
import math
import pathlib
import random
import struct
from fractions import Fraction

HERE = pathlib.Path(__file__).resolve().parent


def f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


def fma(a: float, b: float, c: float) -> float:
    return float(Fraction(a) * Fraction(b) + Fraction(c))


LN2_HEAD = f32(math.log(2.0))
LN2_TAIL = -1.904654299957768e-09
INV_LN2 = 1.4426950408889634
INV_FACT = [1.0 / math.factorial(n) for n in range(14)]


def dp_exp(x: float) -> float:
    if x != x:
        return x
    if x > 709.0:
        return math.inf
    if x < -745.0:
        return 0.0
    k = float(round(x * INV_LN2))  # round half to even, as rint
    hi = x - k * LN2_HEAD
    r = hi - k * LN2_TAIL
    p = INV_FACT[13]
    for n in range(12, -1, -1):
        p = fma(p, r, INV_FACT[n])
    return math.ldexp(p, int(k))


def cuts(col: list[float], max_bin: int):
    vals = sorted(0.0 if v == 0.0 else v for v in col if v == v)
    missing = len(vals) < len(col)
    B = min(max_bin, 255 if missing else 256)
    if not vals:
        return [], missing
    distinct = sorted(set(vals))
    if len(distinct) <= B:
        return distinct[1:], missing
    n = len(vals)
    out: list[float] = []
    for k in range(1, B):
        b = vals[(k * n) // B]
        if b == vals[0] or (out and not b > out[-1]):
            continue
        out.append(b)
    return out, missing


def bin_of(v: float, bounds: list[float]) -> int:
    if v != v:
        return 255
    return sum(1 for c in bounds if c <= v)


def quant_scale(vmax: float, bits: int) -> float:
    if not vmax > 0.0:
        return 1.0
    m, e = math.frexp(vmax)
    e = max(-100, min(100, e))
    return math.ldexp(1.0, bits - e)


def grads(objective: str, K: int, margin: list[list[float]], y: list[float]):
    gh = [[] for _ in range(K)]
    for m, yy in zip(margin, y):
        if objective == "reg:squarederror":
            gh[0].append((f32(m[0] - yy), 1.0))
        elif objective == "binary:logistic":
            p = 1.0 / (1.0 + dp_exp(-m[0]))
            gh[0].append((f32(p - yy), f32(max(p * (1.0 - p), 1e-16))))
        else:
            mx = max(m)
            e = [dp_exp(v - mx) for v in m]
            s = 0.0
            for v in e:
                s = s + v
            for k in range(K):
                pk = e[k] / s
                gh[k].append((f32(pk - (1.0 if k == yy else 0.0)), f32(max(2.0 * pk * (1.0 - pk), 1e-16))))
    return gh


def soft(g: float, a: float) -> float:
    return g - a if g > a else (g + a if g < -a else 0.0)


def score(g, h, p):
    t = soft(g, p["alpha"])
    return (t * t) / (h + p["lambda"])


def grow(bins, F, bounds, nbins, has_missing, gh, p):
    R = len(bins)
    m_g = max(abs(g) for g, _ in gh)
    m_h = max(h for _, h in gh)
    sg, sh = f32(quant_scale(m_g, 17)), f32(quant_scale(m_h, 18))
    q = [(int(round(f32(g * sg))), int(round(f32(h * sh)))) for g, h in gh]
    isg, ish = 1.0 / sg, 1.0 / sh
    nodes = [dict(rows=list(range(R)), depth=0, parent=-1)]
    tree = dict(left=[-1], right=[-1], feature=[0], cond=[0.0], dleft=[0])
    open_ids = [0]
    for depth in range(p["max_depth"]):
        nxt = []
        for nid in open_ids:
            rows = nodes[nid]["rows"]
            G = sum(q[r][0] for r in rows)
            H = sum(q[r][1] for r in rows)
            sp = score(G * isg, H * ish, p)
            best = None
            for f in range(F):
                if nbins[f] < 2:
                    continue
                hist = [[0, 0] for _ in range(256)]
                for r in rows:
                    hist[bins[r][f]][0] += q[r][0]
                    hist[bins[r][f]][1] += q[r][1]
                gm, hm_ = (hist[255] if has_missing[f] else (0, 0))
                gl0 = hl0 = 0
                for b in range(nbins[f] - 1):
                    gl0 += hist[b][0]
                    hl0 += hist[b][1]
                    for d in ((0, 1) if has_missing[f] else (0,)):
                        glq, hlq = gl0 + (gm if d else 0), hl0 + (hm_ if d else 0)
                        GL, HL, GR, HR = glq * isg, hlq * ish, (G - glq) * isg, (H - hlq) * ish
                        if not (HL >= p["mcw"] and HR >= p["mcw"] and HL + p["lambda"] > 0 and HR + p["lambda"] > 0):
                            continue
                        gain = ((score(GL, HL, p) + score(GR, HR, p)) - sp) * 0.5 - p["gamma"]
                        if best is None or gain > best[0]:
                            best = (gain, f, b, d)
            if best is None or not best[0] > 0.0:
                continue
            _, f, b, d = best
            miss = has_missing[f]
            left = [r for r in rows if (d if (miss and bins[r][f] == 255) else bins[r][f] <= b)]
            right = [r for r in rows if not (d if (miss and bins[r][f] == 255) else bins[r][f] <= b)]
            lid, rid = len(nodes), len(nodes) + 1
            nodes += [dict(rows=left, depth=depth + 1, parent=nid), dict(rows=right, depth=depth + 1, parent=nid)]
            for key in ("left", "right", "feature", "cond", "dleft"):
                tree[key] += [-1 if key in ("left", "right") else 0] * 2
            tree["left"][nid], tree["right"][nid] = lid, rid
            tree["feature"][nid], tree["cond"][nid], tree["dleft"][nid] = f, bounds[f][b], d
            nxt += [lid, rid]
        open_ids = nxt
    leaf_of = [0] * R
    for nid, nd in enumerate(nodes):
        if tree["left"][nid] == -1:
            G = sum(q[r][0] for r in nd["rows"]) * isg
            H = sum(q[r][1] for r in nd["rows"]) * ish
            den = H + p["lambda"]
            w = 0.0 if not den > 0 else -soft(G, p["alpha"]) / den
            tree["cond"][nid] = f32(w * p["eta"])
            for r in nd["rows"]:
                leaf_of[r] = nid
    return tree, leaf_of


def train(x, y, objective, K, rounds, p):
    R, F = len(x), len(x[0])
    bounds, has_missing = zip(*(cuts([row[f] for row in x], p["max_bin"]) for f in range(F)))
    nbins = [len(b) + 1 for b in bounds]
    bins = [[bin_of(row[f], bounds[f]) for f in range(F)] for row in x]
    margin = [[0.0] * K for _ in range(R)]
    trees = []
    for _ in range(rounds):
        gh = grads(objective, K, margin, y)
        round_trees = [grow(bins, F, bounds, nbins, has_missing, gh[k], p) for k in range(K)]
        for k, (t, leaf_of) in enumerate(round_trees):
            for r in range(R):
                margin[r][k] = f32(margin[r][k] + t["cond"][leaf_of[r]])
            trees.append(t)
    return dict(bounds=[list(b) for b in bounds], nbins=nbins, has_missing=[int(h) for h in has_missing],
                bins=bins, trees=trees, margin=margin)


def case(name, R, F, objective, K, rounds, seed, nan_frac=0.0, **hp):
    rnd = random.Random(seed)
    x = [[f32(rnd.gauss(0, 1)) for _ in range(F)] for _ in range(R)]
    for row in x:
        if F > 1:
            row[1] = float(rnd.randint(0, 3))  # ties
        for f in range(F):
            if rnd.random() < nan_frac:
                row[f] = math.nan
    if objective == "reg:squarederror":
        y = [f32(2.0 * (row[0] if row[0] == row[0] else 0.0) + rnd.gauss(0, 0.1)) for row in x]
    elif objective == "binary:logistic":
        y = [1.0 if (row[0] if row[0] == row[0] else 0.0) + 0.3 * rnd.gauss(0, 1) > 0 else 0.0 for row in x]
    else:
        y = [float(rnd.randint(0, K - 1)) for _ in x]
    p = dict(max_depth=hp.get("max_depth", 3), max_bin=hp.get("max_bin", 256), eta=hp.get("eta", 0.3),
             alpha=hp.get("alpha", 0.0), gamma=hp.get("gamma", 0.0), mcw=hp.get("mcw", 1.0),
             **{"lambda": hp.get("reg_lambda", 1.0)})
    out = train(x, y, objective, K, rounds, p)
    doc = dict(name=name, objective=objective, num_class=K, rounds=rounds, params=p,
               x=[[None if v != v else v for v in row] for row in x], y=y, expected=out)
    (HERE / f"{name}.json").write_text(json.dumps(doc))


if __name__ == "__main__":
    case("logistic_nan", 64, 3, "binary:logistic", 1, 3, 1, nan_frac=0.15, max_depth=3)
    case("softmax_k3", 48, 4, "multi:softmax", 3, 2, 2, max_depth=2, mcw=0.1)
    case("squared_quantile", 40, 2, "reg:squarederror", 1, 3, 3, max_bin=4, alpha=0.3, gamma=0.05, mcw=0.5,
         reg_lambda=2.0, max_depth=2)
    case("squared_deep", 30, 3, "reg:squarederror", 1, 2, 4, max_depth=5, mcw=0.0, reg_lambda=0.5, eta=1.0)
