"""Device radius graph (ops/csrc/graph.cu) against the host cell list: same edges, same order."""
import numpy as np
import pytest

from maloq_b200.data import structures
from maloq_b200.data.graph import radius_graph
from maloq_b200.data.graph_gpu import radius_graph_device

pytestmark = pytest.mark.gpu


def _check(pos, cutoff, cell=None, targets=None):
    src, dst, vec = radius_graph(pos, cutoff, cell)
    if targets is not None:
        keep = np.isin(dst, targets)
        remap = np.full(len(pos), -1)
        remap[targets] = np.arange(len(targets))
        src, dst, vec = src[keep], remap[dst[keep]], vec[keep]
        o = np.lexsort((src, dst))
        src, dst, vec = src[o], dst[o], vec[o]
    s, d, v, ptr = radius_graph_device(pos, cutoff, cell, targets)
    assert np.array_equal(s.cpu().numpy(), src)
    assert np.array_equal(d.cpu().numpy(), dst)
    assert np.allclose(v.cpu().numpy(), vec, atol=1e-12)
    n_t = len(pos) if targets is None else len(targets)
    assert np.array_equal(ptr.cpu().numpy(), np.concatenate([[0], np.cumsum(np.bincount(dst, minlength=n_t))]))


def test_periodic_sio2():
    rng = np.random.default_rng(0)
    s = structures.amorphous_sio2(rng, 3000)
    _check(s.pos, 8.0, s.cell)


def test_periodic_small_cell_dedupes_images():
    rng = np.random.default_rng(1)
    cell = np.array([10.5, 12.0, 17.0])  # 1-2 cells per axis at a 5 A cutoff
    _check(rng.uniform(0, 1, (200, 3)) * cell, 5.0, cell)


def test_open_molecule_and_target_subset():
    rng = np.random.default_rng(2)
    s = structures.random_large_molecule(rng)
    _check(s.pos, 6.0)
    slab = structures.si_slab_with_oxide(rng, 4000)
    targets = np.flatnonzero(slab.pos[:, 0] < slab.cell[0] / 2)
    _check(slab.pos, 8.0, slab.cell, targets)
