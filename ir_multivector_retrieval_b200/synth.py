"""Seeded synthetic token corpus with the shape of the BASELINE configs.

Each vector is ``normalize(anchor + 0.35 * N(0, I))``; anchors are
``n_anchors`` unit vectors uniform on the sphere and a token's id is the
rank of its anchor, drawn Zipf(``zipf_s``) over the anchors. Documents hold
about ``tokens_per_doc`` tokens. This stands in for the reference's private
Jira corpus (jina-colbert-v2-64 embeddings); no public benchmark data is
involved.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Corpus:
    token_ids: np.ndarray  # (n,) uint32
    vectors: np.ndarray  # (n, dim) float32, unit rows
    doc_offsets: np.ndarray  # (n_docs + 1,) uint64
    anchors: np.ndarray  # (n_anchors, dim) float32

    @property
    def n(self) -> int:
        return int(self.token_ids.shape[0])

    @property
    def dim(self) -> int:
        return int(self.vectors.shape[1])


def _normalize_rows(x: np.ndarray) -> np.ndarray:
    n = np.sqrt(np.einsum("ij,ij->i", x, x, dtype=np.float64)).astype(np.float32)
    n[n == 0] = 1.0
    return (x / n[:, None]).astype(np.float32)


def make_corpus(n_tokens: int, dim: int = 64, *, n_anchors: int = 19221, zipf_s: float = 1.1,
                noise: float = 0.35, seed: int = 42, tokens_per_doc: int = 57,
                chunk: int = 1 << 20) -> Corpus:
    rng = np.random.default_rng(seed)
    anchors = _normalize_rows(rng.standard_normal((n_anchors, dim), dtype=np.float32))
    w = 1.0 / np.power(np.arange(1, n_anchors + 1, dtype=np.float64), zipf_s)
    cdf = np.cumsum(w / w.sum())
    ids = np.searchsorted(cdf, rng.random(n_tokens), side="right").astype(np.uint32)
    np.minimum(ids, n_anchors - 1, out=ids)
    vec = np.empty((n_tokens, dim), dtype=np.float32)
    for s in range(0, n_tokens, chunk):
        e = min(n_tokens, s + chunk)
        g = rng.standard_normal((e - s, dim), dtype=np.float32)
        vec[s:e] = _normalize_rows(anchors[ids[s:e]] + np.float32(noise) * g)
    n_docs = max(1, n_tokens // tokens_per_doc)
    cuts = np.sort(rng.choice(np.arange(1, n_tokens), size=n_docs - 1, replace=False)) if n_docs > 1 else []
    doc_offsets = np.concatenate([[0], cuts, [n_tokens]]).astype(np.uint64)
    return Corpus(token_ids=ids, vectors=vec, doc_offsets=doc_offsets, anchors=anchors)


def anchor_residuals(c: Corpus) -> np.ndarray:
    """Unit residuals of each vector from its token's anchor: the input
    shape PQ training sees (normalised residuals, storage.zig:255-278),
    with the anchor standing in for the token's TAC centroid."""
    return _normalize_rows(c.vectors - c.anchors[c.token_ids])


def unit_rows(n: int, dim: int, seed: int = 0) -> np.ndarray:
    """n unit-norm Gaussian rows (float32)."""
    rng = np.random.default_rng(seed)
    return _normalize_rows(rng.standard_normal((n, dim), dtype=np.float32))


def device_residuals(n_tokens: int, dim: int, *, n_anchors: int = 19221, zipf_s: float = 1.1, noise: float = 0.35,
                     seed: int = 42, device: str = "cuda", row0: int = 0, n_rows: int | None = None,
                     chunk: int = 1 << 22):
    """The same generator run on the GPU for corpora too large to make on the
    host (BASELINE configs[3] and [4]): anchors uniform on the sphere, token
    id = Zipf(zipf_s) rank, vector = normalize(anchor + noise N(0, I)), and
    the PQ input row = normalize(vector - anchor), the unit residual from
    the token's anchor (standing in for its TAC centroid). Rows
    [row0, row0 + n_rows) of the n_tokens-row corpus are made; each block of
    `chunk` rows has its own seeded torch Philox stream, so any shard of the
    corpus comes out the same whichever process makes it. The values differ
    from make_corpus at equal seeds; the distributions are the same. Returns
    (residuals n_rows x dim f32, token ids int64), both on `device`."""
    import torch

    n_rows = n_tokens - row0 if n_rows is None else n_rows
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    anchors = torch.randn((n_anchors, dim), generator=g, device=device, dtype=torch.float32)
    anchors /= anchors.norm(dim=1, keepdim=True)
    w = 1.0 / torch.arange(1, n_anchors + 1, device=device, dtype=torch.float64) ** zipf_s
    cdf = torch.cumsum(w / w.sum(), 0)
    res = torch.empty((n_rows, dim), device=device, dtype=torch.float32)
    ids = torch.empty(n_rows, device=device, dtype=torch.int64)
    lo, hi = row0, row0 + n_rows
    for c in range(lo // chunk, (hi + chunk - 1) // chunk):
        c0, c1 = c * chunk, min(n_tokens, (c + 1) * chunk)
        gc = torch.Generator(device=device)
        gc.manual_seed(int(seed) * 1_000_003 + 7 + c)
        u = torch.rand(c1 - c0, generator=gc, device=device, dtype=torch.float64)
        t = torch.clamp(torch.searchsorted(cdf, u, right=True), max=n_anchors - 1)
        v = anchors[t] + noise * torch.randn((c1 - c0, dim), generator=gc, device=device, dtype=torch.float32)
        v /= v.norm(dim=1, keepdim=True).clamp_min(1e-30)
        r = v - anchors[t]
        nr = r.norm(dim=1, keepdim=True)
        r = torch.where(nr > 0, r / nr.clamp_min(1e-30), r)
        a, b = max(lo, c0), min(hi, c1)
        res[a - lo:b - lo] = r[a - c0:b - c0]
        ids[a - lo:b - lo] = t[a - c0:b - c0]
        del u, t, v, r, nr
    return res, ids
