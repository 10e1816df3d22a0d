"""Backbone embedding dumps and their analysis.

``dump(folder, index, emb, batch)`` writes ``embeddings_{index}.npz`` (node embeddings
[N, (L+1)^2, C], edge embeddings if present, edge attributes, positions, atomic numbers);
:func:`invariant_features` turns equivariant embeddings into rotation-invariant rows (the
l = 0 channels and the norm over m of every l > 0 channel), which :func:`project` (PCA or
t-SNE) and :func:`cluster` (k-means) use.  Reference: ``splittrainer.py:1235-1267`` (dumps)
and ``scripts/visualize_backbone_embeddings.py`` (projections, clustering).

    python -m maloq_b200.analysis.embeddings outputs/embeddings --method pca --clusters 6
"""

from __future__ import annotations

import argparse
import glob
import os

import numpy as np


def dump(folder, index, emb, batch):
    os.makedirs(folder, exist_ok=True)
    arrays = {"node_embeddings": emb["node_embeddings"], "edge_attr": batch.edge_attr, "pos": batch.pos,
              "atomic_numbers": batch.atomic_numbers}
    if emb.get("edge_embeddings") is not None:
        arrays["edge_embeddings"] = emb["edge_embeddings"]
    path = os.path.join(folder, f"embeddings_{index}.npz")
    np.savez(path, **{k: v.detach().float().cpu().numpy() if hasattr(v, "detach") else np.asarray(v)
                      for k, v in arrays.items()})
    return path


def load(folder, key="node_embeddings"):
    """Concatenated ``key`` rows and atomic numbers of every dump in ``folder`` (index order)."""
    files = sorted(glob.glob(os.path.join(folder, "embeddings_*.npz")),
                   key=lambda p: int(os.path.basename(p)[11:-4]))
    xs, zs = [], []
    for f in files:
        d = np.load(f)
        xs.append(d[key])
        zs.append(d["atomic_numbers"] if key == "node_embeddings" else np.zeros(len(d[key]), np.int64))
    return np.concatenate(xs), np.concatenate(zs)


def invariant_features(x):
    """[N, (L+1)^2, C] -> [N, (L+1) * C]: l = 0 channels, then |x_l| over m for l = 1..L."""
    x = np.asarray(x)
    L = int(round(np.sqrt(x.shape[1]))) - 1
    feats = [x[:, 0]]
    for l in range(1, L + 1):
        feats.append(np.linalg.norm(x[:, l * l:(l + 1) * (l + 1)], axis=1))
    return np.concatenate(feats, axis=1)


def project(features, method="pca", dim=2, seed=0):
    from sklearn.decomposition import PCA
    from sklearn.preprocessing import StandardScaler

    f = StandardScaler().fit_transform(features)
    if method == "pca":
        return PCA(n_components=dim, random_state=seed).fit_transform(f)
    if method == "tsne":
        from sklearn.manifold import TSNE

        pre = PCA(n_components=min(50, f.shape[1], len(f)), random_state=seed).fit_transform(f)
        return TSNE(n_components=dim, random_state=seed, init="pca",
                    perplexity=min(30.0, max(2.0, (len(f) - 1) / 3))).fit_transform(pre)
    raise ValueError(f"unknown projection {method!r} (pca, tsne)")


def cluster(features, k, seed=0):
    from sklearn.cluster import KMeans
    from sklearn.preprocessing import StandardScaler

    return KMeans(n_clusters=k, random_state=seed, n_init=10).fit_predict(StandardScaler().fit_transform(features))


def main(argv=None):
    ap = argparse.ArgumentParser(description="project and cluster dumped backbone embeddings")
    ap.add_argument("folder")
    ap.add_argument("--method", default="pca", choices=["pca", "tsne"])
    ap.add_argument("--clusters", type=int, default=0)
    ap.add_argument("--out", default=None, help="CSV path (default <folder>/projection_<method>.csv)")
    a = ap.parse_args(argv)
    x, z = load(a.folder)
    f = invariant_features(x)
    p = project(f, a.method)
    lab = cluster(f, a.clusters) if a.clusters else np.zeros(len(f), np.int64)
    out = a.out or os.path.join(a.folder, f"projection_{a.method}.csv")
    np.savetxt(out, np.column_stack([z, p, lab]), delimiter=",", header="atomic_number,x,y,cluster", comments="",
               fmt=["%d", "%.6g", "%.6g", "%d"])
    print(out)
    return out


if __name__ == "__main__":
    main()
