"""Whole ops and a model training step on the CUDA kernel sources, run on the CPU emulator
(``tests/emulated_extension.py``): the label conversions and basis transform (``labels.cu``), the
device radius graph (``graph.cu``), the edge rotation and fused loss (``misc.cu``) and the
model's kernel path (edge frame, norms, gates, head gate) against the PyTorch definitions.  The
kernels are built with the index checks on (``MALOQ_BOUNDS_CHECK``); every test also asserts
that no kernel recorded an error code."""
import numpy as np
import pytest
import torch

from tests.emulated_extension import load_libraries, use_emulated_extension


@pytest.fixture(scope="module")
def libs(tmp_path_factory):
    libs = load_libraries(tmp_path_factory.mktemp("emu_ops"), defines=("MALOQ_BOUNDS_CHECK=1",))
    if libs is None:
        pytest.skip("needs g++ and the CUDA headers")
    return libs


def _labels_case(kind, n_mol, dtype, seed=0):
    from maloq_b200.data import datasets

    labeler = datasets.labeler_for(kind, "cpu")
    samples = datasets.build_samples(kind, n_mol, seed=seed)
    tbl = labeler.table
    ptrs, pts, n = [0], [], 0
    for s in samples:
        rows, cols = labeler.pairs(s)
        nz = tbl.norb[tbl.z_to_type[s.z]]
        for sz in nz[rows] * nz[cols]:
            n += int(sz)
            ptrs.append(n)
        pts.append(tbl.pair_type(s.z[rows], s.z[cols]))
    g = torch.Generator().manual_seed(seed)
    data = torch.randn(n, generator=g, dtype=torch.float64).to(dtype)
    return labeler, data, torch.tensor(ptrs), torch.as_tensor(np.concatenate(pts), dtype=torch.long), n


@pytest.mark.parametrize("kind,n_mol,dtype", [("druglike", 1, torch.float32), ("druglike", 1, torch.float64),
                                              ("large", 1, torch.float32)])
def test_label_ops_on_emulated_kernels(monkeypatch, libs, kind, n_mol, dtype):
    from maloq_b200.ops import basis_transform as bt
    from maloq_b200.ops import labels as lab

    labeler, data, ptr, pt, n = _labels_case(kind, n_mol, dtype)
    pos, T = labeler.pos_t.cpu(), labeler.transform
    ref_lab = lab._ref_m2l(data, ptr, pt, pos)
    ref_c = ref_lab.double() @ T.W_global_inv.double()
    x = ref_c.to(dtype)
    ref_h = x.double() @ T.W_global.double()
    ref_d = lab._ref_l2m(ref_h, ptr, pt, pos, n)
    ext = use_emulated_extension(monkeypatch, libs)
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    got_lab = lab.matrix_to_labels(data, ptr, pt, pos)
    assert torch.equal(got_lab, ref_lab)
    assert torch.equal(lab.labels_to_matrix(got_lab, ptr, pt, pos, n), lab._ref_l2m(ref_lab, ptr, pt, pos, n))
    for got, ref in ((lab.blocks_to_coupled(data, ptr, pt, pos, T), ref_c),
                     (bt.apply_transform(x, T, inverse=False), ref_h),
                     (lab.coupled_to_blocks(x, ptr, pt, pos, T, n), ref_d)):
        got = got.double()
        assert (got - ref).abs().max() <= tol * max(1.0, ref.abs().max().item())
    assert ext.emulated_calls["basis_rows"] == 5
    assert ext.emulated_error_word() == 0


def test_label_gather_with_a_bad_pair_type_records_an_error(monkeypatch, libs):
    """A pair type outside the position table skips the access and records the bounds code."""
    from maloq_b200.ops import labels as lab

    labeler, data, ptr, pt, n = _labels_case("druglike", 1, torch.float32)
    pt = pt.clone()
    pt[0] = labeler.pos_t.shape[0] + 3
    ext = use_emulated_extension(monkeypatch, libs)
    out = lab.matrix_to_labels(data, ptr, pt, labeler.pos_t.cpu())
    assert ext.emulated_error_word() == 5  # ERR_BOUNDS
    assert torch.all(out[0] == 0)
