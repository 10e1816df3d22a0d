"""Label kernels (ops/csrc/labels.cu) against the PyTorch definitions: block-sparse <-> label
rows, the block-diagonal basis transform, and the fused gather/scatter + transform forms."""
import numpy as np
import pytest
import torch

from maloq_b200.data import datasets
from maloq_b200.ops import basis_transform as bt
from maloq_b200.ops import labels as lab
from maloq_b200.ops.labels import _ref_l2m, _ref_m2l

pytestmark = pytest.mark.gpu


def _case(kind, n_mol, dtype, seed=0):
    labeler = datasets.labeler_for(kind, "cuda")
    samples = datasets.build_samples(kind, n_mol, seed=seed)
    tbl = labeler.table
    ptrs, pts, n = [0], [], 0
    for s in samples:
        rows, cols = labeler.pairs(s)
        nz = tbl.norb[tbl.z_to_type[s.z]]
        sizes = nz[rows] * nz[cols]
        for sz in sizes:
            n += int(sz)
            ptrs.append(n)
        pts.append(tbl.pair_type(s.z[rows], s.z[cols]))
    g = torch.Generator().manual_seed(seed)
    data = torch.randn(n, generator=g, dtype=torch.float64)
    ptr = torch.tensor(ptrs, dtype=torch.long)  # block offsets, len rows + 1
    pt = torch.as_tensor(np.concatenate(pts), dtype=torch.long)
    return labeler, data.to(dtype), ptr, pt, n


@pytest.mark.parametrize("kind", ["druglike", "large"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_blocks_labels_roundtrip_and_transform(kind, dtype):
    labeler, data, ptr, pt, n = _case(kind, 3, dtype)
    pos = labeler.pos_t.cpu()
    T = labeler.transform
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    # plain gather / scatter
    ref_lab = _ref_m2l(data, ptr, pt, pos)
    got_lab = lab.matrix_to_labels(data.cuda(), ptr.cuda(), pt.cuda(), pos.cuda()).cpu()
    assert torch.equal(got_lab, ref_lab)
    got_back = lab.labels_to_matrix(got_lab.cuda(), ptr.cuda(), pt.cuda(), pos.cuda(), n).cpu()
    assert torch.equal(got_back, _ref_l2m(ref_lab, ptr, pt, pos, n))
    # fused gather + get_net_out vs fp64 dense matmul
    W_inv = T.W_global_inv.cpu().double()
    ref_c = ref_lab.double() @ W_inv
    got_c = lab.blocks_to_coupled(data.cuda(), ptr.cuda(), pt.cuda(), pos.cuda(), T).cpu().double()
    assert (got_c - ref_c).abs().max() <= tol * max(1.0, ref_c.abs().max().item())
    # dense transform both ways
    x = ref_c.to(dtype)
    got_h = bt.apply_transform(x.cuda(), T, inverse=False).cpu().double()
    ref_h = x.double() @ T.W_global.cpu().double()
    assert (got_h - ref_h).abs().max() <= tol * max(1.0, ref_h.abs().max().item())
    # fused get_H + scatter inverts the gather path on the stored positions
    got_d = lab.coupled_to_blocks(x.cuda(), ptr.cuda(), pt.cuda(), pos.cuda(), T, n).cpu().double()
    ref_d = _ref_l2m(ref_h, ptr, pt, pos, n)
    assert (got_d - ref_d).abs().max() <= tol * max(1.0, ref_d.abs().max().item())
    # the CG matrices are stored in fp32, so the round trip is exact to ~1e-7 relative
    assert (got_d - data.double()).abs().max() <= 1e-5 * max(1.0, data.abs().max().item())


def test_labeler_targets_match_cpu_path():
    """FockLabeler on CUDA (fused kernels) gives the CPU (dense matmul) coupled labels."""
    labeler_gpu = datasets.labeler_for("druglike", "cuda")
    labeler_cpu = datasets.labeler_for("druglike", "cpu")
    s = datasets.build_samples("druglike", 1, seed=5)[0]
    from maloq_b200.data.labels import BlockSparseMatrix, orbital_offsets

    rows, cols = labeler_cpu.pairs(s)
    orb = orbital_offsets(s.z, labeler_cpu.table)
    rng = np.random.default_rng(0)
    M = rng.standard_normal((orb[-1], orb[-1]))
    bsm = BlockSparseMatrix.from_dense(M.astype(np.float32), rows, cols, orb)
    n_g, e_g = labeler_gpu.labels_from_blocks(s, bsm)
    n_c, e_c = labeler_cpu.labels_from_blocks(s, bsm)
    assert torch.allclose(n_g.cpu(), n_c, atol=1e-5, rtol=1e-5)
    assert torch.allclose(e_g.cpu(), e_c, atol=1e-5, rtol=1e-5)
    back = labeler_gpu.blocks_from_labels(s, n_g, e_g)
    assert np.allclose(back.data, bsm.data, atol=1e-4)


def test_basis_transform_gradient_matches_matmul():
    labeler = datasets.labeler_for("druglike", "cuda")
    T = labeler.transform
    x = torch.randn(50, T.dim, device="cuda", requires_grad=True)
    w = torch.randn(50, T.dim, device="cuda")
    (bt.apply_transform(x, T, inverse=False) * w).sum().backward()
    ref = w @ T.W_global.to("cuda").float().t()
    assert (x.grad - ref).abs().max() <= 1e-5 * max(1.0, ref.abs().max().item())
