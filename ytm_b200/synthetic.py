"""Seeded synthetic workloads standing in for the benchmark configurations
(no datasets are available offline).  Each returns raw u32 inputs
[N, D0*D1*D2] (0/1) and integer labels, in the layout the reference's
scripts feed to `fit` (e.g. test/cutm/mnist/mnist_conv.py:43-46).

MODELS maps each configuration to the reference constructor arguments.
"""
from __future__ import annotations

import numpy as np

MODELS = {
    # 1. vanilla: 2000 clauses per class, non-coalesced, batch 1
    "c1": dict(number_of_clauses_per_class=2000, T=50, s=10.0, dim=(28, 28, 1), n_classes=10, coalesced=False),
    # 2. coalesced: 10k shared clauses, mini-batch 256
    "c2": dict(number_of_clauses_per_class=10000, T=1000, s=15.0, dim=(28, 28, 1), n_classes=10, coalesced=True),
    # 3. convolutional 28x28, 10x10 patches
    "c3": dict(number_of_clauses_per_class=8000, T=10000, s=5.0, dim=(28, 28, 1), n_classes=10, patch_dim=(10, 10),
               encode_loc=True),
    # 4. convolutional 32x32x(3 channels x 8 thermometer levels), 10x10 patches
    "c4": dict(number_of_clauses_per_class=20000, T=15000, s=10.0, dim=(32, 32, 24), n_classes=10,
               patch_dim=(10, 10)),
    # 5. large: 65536 shared clauses, 16384 features, 100 classes, 12-bit states
    "c5": dict(number_of_clauses_per_class=65536, T=20000, s=20.0, dim=(16384, 1, 1), n_classes=100,
               number_of_ta_states=4096),
}
# pytm's own rules (src/pytm/base.py) at the 2000-clause, 784-feature size the
# reference's numpy TM was timed on: 2000 shared clauses, pytm's default 256
# states (0..255 = this engine's number_of_ta_states 255), batch 1
MODELS["p1"] = dict(number_of_clauses_per_class=2000, T=50, s=10.0, dim=(28, 28, 1), n_classes=10, coalesced=True,
                    number_of_ta_states=255, rules="pytm")
BATCH = {"c1": 1, "c2": 256, "c3": 1, "c4": 1, "c5": 1024, "p1": 1}
SEEDS = {"c1": 1001, "c2": 1002, "c3": 1003, "c4": 1004, "c5": 1005, "p1": 1001}


def prototypes(N, seed=1001, n_classes=10, n_features=784, p_one=0.2, p_flip=0.05):
    """Configs 1-2: one random prototype bit-vector per class (p=0.2 ones);
    each sample flips each prototype bit with p=0.05."""
    rng = np.random.default_rng(seed)
    protos = rng.random((n_classes, n_features)) < p_one
    y = rng.integers(0, n_classes, N)
    flips = rng.random((N, n_features)) < p_flip
    X = (protos[y] ^ flips).astype(np.uint32)
    return X, y.astype(np.uint32)


def glyphs(N, seed=1003, n_classes=10, size=28, glyph=5, p_noise=0.02):
    """Config 3: one 5x5 Bernoulli(0.5) glyph per class OR-ed at a uniform
    offset onto Bernoulli(0.02) noise."""
    rng = np.random.default_rng(seed)
    g = rng.random((n_classes, glyph, glyph)) < 0.5
    y = rng.integers(0, n_classes, N)
    img = rng.random((N, size, size)) < p_noise
    oy = rng.integers(0, size - glyph + 1, N)
    ox = rng.integers(0, size - glyph + 1, N)
    for i in range(N):
        img[i, oy[i]:oy[i] + glyph, ox[i]:ox[i] + glyph] |= g[y[i]]
    return img.reshape(N, -1).astype(np.uint32), y.astype(np.uint32)


def thermometer_rgb(X, levels=8):
    """ThermometerBinarizer.binarize_rgb semantics (tm_utils/binarizer.py:17-21):
    bit c*levels+j of a pixel is X[..., c] >= (j+1)*255/(levels+1)."""
    thr = (np.arange(1, levels + 1) * 255 / (levels + 1)).reshape(1, 1, 1, 1, levels)
    out = X[..., None] >= thr
    return out.reshape(X.shape[0], X.shape[1], X.shape[2], X.shape[3] * levels).astype(np.uint32)


def blobs(N, seed=1004, n_classes=10, size=32, sigma=0.15):
    """Config 4: per class a seeded mixture of 3 Gaussian colour blobs over
    uniform noise, x255, thermometer-encoded to 8 bits per channel."""
    rng = np.random.default_rng(seed)
    centres = rng.random((n_classes, 3, 2))
    colours = rng.random((n_classes, 3, 3))
    y = rng.integers(0, n_classes, N)
    yy, xx = np.meshgrid(np.linspace(0, 1, size), np.linspace(0, 1, size), indexing="ij")
    out = np.empty((N, size * size * 3 * 8), np.uint32)
    for s in range(0, N, 1024):
        e = min(N, s + 1024)
        img = rng.random((e - s, size, size, 3)) * 0.5
        for b in range(3):
            c = centres[y[s:e], b]
            d2 = (yy[None] - c[:, 0, None, None]) ** 2 + (xx[None] - c[:, 1, None, None]) ** 2
            img += np.exp(-d2 / (2 * sigma ** 2))[..., None] * colours[y[s:e], b][:, None, None, :]
        img = np.clip(img, 0, 1) * 255
        out[s:e] = thermometer_rgb(img).reshape(e - s, -1)
    return out, y.astype(np.uint32)


def rules(N, seed=1005, n_classes=100, n_features=16384, density=0.01, rules_per_class=10, rule_len=8):
    """Config 5: sparse Bernoulli(0.01) features; each sample draws a class and
    one of its 10 planted 8-literal rules and forces those literals."""
    rng = np.random.default_rng(seed)
    feat = rng.integers(0, n_features, (n_classes, rules_per_class, rule_len))
    pol = rng.random((n_classes, rules_per_class, rule_len)) < 0.5
    y = rng.integers(0, n_classes, N)
    r = rng.integers(0, rules_per_class, N)
    X = (rng.random((N, n_features)) < density)
    rows = np.repeat(np.arange(N), rule_len)
    X[rows, feat[y, r].reshape(-1)] = pol[y, r].reshape(-1)
    return X.astype(np.uint32), y.astype(np.uint32)


def rules_torch(N, seed, device, n_classes=100, n_features=16384, density=0.01, rules_per_class=10, rule_len=8,
                rule_seed=1005):
    """Config 5 generated on the GPU (for the 2^20-sample inference run, 64 GB
    as host u32): the same planted rules as rules(rule_seed) (the rule table is
    drawn with numpy), Bernoulli(density) background and labels from a torch
    generator seeded with `seed`.  Returns int32 [N, n_features] 0/1 on device."""
    import torch
    rng = np.random.default_rng(rule_seed)
    feat = torch.from_numpy(rng.integers(0, n_features, (n_classes, rules_per_class, rule_len))).to(device)
    pol = torch.from_numpy(rng.random((n_classes, rules_per_class, rule_len)) < 0.5).to(device)
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    y = torch.randint(0, n_classes, (N,), generator=g, device=device)
    r = torch.randint(0, rules_per_class, (N,), generator=g, device=device)
    X = (torch.rand((N, n_features), generator=g, device=device) < density).to(torch.int32)
    rows = torch.arange(N, device=device).repeat_interleave(rule_len)
    X[rows, feat[y, r].reshape(-1)] = pol[y, r].reshape(-1).to(torch.int32)
    return X


def make(name, N, seed=None):
    seed = SEEDS[name] if seed is None else seed
    if name in ("c1", "c2", "p1"):
        return prototypes(N, seed)
    if name == "c3":
        return glyphs(N, seed)
    if name == "c4":
        return blobs(N, seed)
    if name == "c5":
        return rules(N, seed)
    raise KeyError(name)
