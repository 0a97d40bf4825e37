"""Product-quantised retrieval (reference src/omnicoder/inference/retrieval_pq.py:1-344).

Documents -> TF-IDF vectors (scikit-learn) -> optional dense projection ->
product quantisation: the vector is split into M sub-vectors, each replaced by
the index of its nearest centroid among K (k-means per subspace).  Search uses
asymmetric distances: per query, an [M, K] table of squared distances from
the query's sub-vectors to every centroid, summed along each document's codes.
"""
from __future__ import annotations

import numpy as np


def _kmeans(x: np.ndarray, k: int, iters: int = 20, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    k = min(k, len(x))
    c = x[rng.choice(len(x), k, replace=False)].copy()
    for _ in range(iters):
        d = ((x[:, None, :] - c[None]) ** 2).sum(-1)
        a = d.argmin(1)
        for j in range(k):
            m = a == j
            if m.any():
                c[j] = x[m].mean(0)
    return c


class PQRetriever:
    def __init__(self, n_subspaces: int = 8, n_centroids: int = 64, dim: int = 256, seed: int = 0):
        self.M, self.K, self.dim, self.seed = n_subspaces, n_centroids, dim, seed

    def fit(self, docs: list[str]) -> "PQRetriever":
        from sklearn.feature_extraction.text import TfidfVectorizer
        self.docs = list(docs)
        self.vec = TfidfVectorizer(max_features=20000)
        X = self.vec.fit_transform(self.docs).astype(np.float32)
        F = X.shape[1]
        rng = np.random.default_rng(self.seed)
        d = max(self.M, (min(self.dim, F) // self.M) * self.M)
        self.proj = (rng.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
        Z = np.asarray(X @ self.proj)
        Z /= np.linalg.norm(Z, axis=1, keepdims=True) + 1e-9
        self.sub = d // self.M
        self.codebooks, codes = [], []
        for m in range(self.M):
            part = Z[:, m * self.sub:(m + 1) * self.sub]
            cb = _kmeans(part, self.K, seed=self.seed + m)
            self.codebooks.append(cb)
            codes.append(((part[:, None] - cb[None]) ** 2).sum(-1).argmin(1))
        self.codes = np.stack(codes, 1)            # [n_docs, M]
        return self

    def _embed(self, q: str) -> np.ndarray:
        z = np.asarray(self.vec.transform([q]).astype(np.float32) @ self.proj)[0]
        return z / (np.linalg.norm(z) + 1e-9)

    def search(self, query: str, k: int = 5) -> list[tuple[int, float, str]]:
        z = self._embed(query)
        table = np.stack([((self.codebooks[m] - z[m * self.sub:(m + 1) * self.sub]) ** 2).sum(-1)
                          for m in range(self.M)])  # [M, K]
        dist = table[np.arange(self.M)[None, :], self.codes].sum(1)
        top = np.argsort(dist)[:k]
        return [(int(i), float(dist[i]), self.docs[i]) for i in top]

    def budget_profile(self) -> dict:
        """Bytes the index keeps resident: codes (1 byte per sub-vector when K <= 256), codebooks,
        the projection and the vocabulary's idf weights."""
        code_b = 1 if self.K <= 256 else 2
        return {"docs": len(self.docs), "subspaces": self.M, "centroids": self.K, "dim": self.sub * self.M,
                "codes_bytes": int(self.codes.shape[0] * self.M * code_b),
                "codebooks_bytes": int(sum(c.size for c in self.codebooks) * 4),
                "projection_bytes": int(self.proj.size * 4),
                "idf_bytes": int(len(self.vec.idf_) * 4)}

    def save(self, out_dir: str) -> None:
        """Arrays in `pq.npz`, vocabulary / settings / documents in `pq.json` (no pickles)."""
        import json
        import os
        os.makedirs(out_dir, exist_ok=True)
        np.savez(os.path.join(out_dir, "pq.npz"), proj=self.proj, codes=self.codes,
                 codebooks=np.stack(self.codebooks), idf=self.vec.idf_.astype(np.float64))
        with open(os.path.join(out_dir, "pq.json"), "w", encoding="utf-8") as f:
            json.dump({"M": self.M, "K": self.K, "dim": self.dim, "seed": self.seed, "sub": self.sub,
                       "vocabulary": {k: int(v) for k, v in self.vec.vocabulary_.items()}, "docs": self.docs}, f)

    @classmethod
    def load(cls, out_dir: str) -> "PQRetriever":
        import json
        import os
        from sklearn.feature_extraction.text import TfidfVectorizer
        with open(os.path.join(out_dir, "pq.json"), encoding="utf-8") as f:
            meta = json.load(f)
        arr = np.load(os.path.join(out_dir, "pq.npz"))
        r = cls(meta["M"], meta["K"], meta["dim"], meta["seed"])
        r.sub, r.docs = meta["sub"], meta["docs"]
        r.vec = TfidfVectorizer(vocabulary=meta["vocabulary"])
        r.vec.idf_ = arr["idf"]
        r.proj, r.codes = arr["proj"], arr["codes"]
        r.codebooks = list(arr["codebooks"])
        return r
