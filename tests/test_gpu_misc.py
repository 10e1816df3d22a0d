"""Edge rotation, fused loss and column-sum kernels vs their PyTorch definitions."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("lmax,mmax", [(4, 2), (4, 4), (6, 2), (2, 1)])
def test_edge_rotation_matches_reference(cuda_device, lmax, mmax):
    from maloq_b200.core import sph
    from maloq_b200.models.so3 import CoefficientMapping
    from maloq_b200.ops import misc_native
    from maloq_b200.ops import reference as R

    torch.manual_seed(0)
    v = torch.randn(5000, 3, device=cuda_device, dtype=torch.float64)
    v[:3] = torch.tensor([[0.0, 1.0, 0.0], [0.0, -1.0, 0.0], [1.0, 0.0, 0.0]], dtype=torch.float64)
    mp = CoefficientMapping(lmax, mmax).to(cuda_device)
    Js = [j.to(cuda_device) for j in sph.J_matrices(lmax)]
    ref = R.edge_rotation(v, lmax, mmax, Js, mp).float()
    out = misc_native.edge_rotation(v.float(), lmax, mmax, Js, mp)
    assert (out - ref).abs().max().item() < 2e-4


@pytest.mark.parametrize("name", ["rmse_mse_padded_loss", "mse_padded_loss", "l1_padded_loss", "combined_padded_loss"])
def test_fused_fock_loss_matches_reference(cuda_device, name):
    from maloq_b200.ops import misc_native
    from maloq_b200.ops import reference as R
    from maloq_b200.train import loss as L

    torch.manual_seed(1)
    D, T = 324, 4
    mask = torch.rand(T * T, D, device=cuda_device) > 0.3
    no = torch.randn(200, D, device=cuda_device, requires_grad=True)
    eo = torch.randn(3000, D, device=cuda_device, requires_grad=True)
    nt, et = torch.randn(200, D, device=cuda_device), torch.randn(3000, D, device=cuda_device)
    npt = torch.randint(0, T * T, (200,), device=cuda_device)
    ept = torch.randint(0, T * T, (3000,), device=cuda_device)
    out = misc_native.fock_loss(no, eo, nt, et, mask, npt, ept, name)
    ref = R.fock_loss(no, eo, nt, et, mask[npt], mask[ept], L.get_loss(name))
    for a, b in zip(out, ref):
        assert abs(a.item() - b.item()) <= 1e-5 * abs(b.item()) + 1e-7
    ga = torch.autograd.grad(out[2], [no, eo])
    gr = torch.autograd.grad(ref[2], [no, eo])
    for a, b in zip(ga, gr):
        assert (a - b).abs().max().item() <= 1e-5 * b.abs().max().item() + 1e-9


def test_peer_barrier_timeout_reports_error_and_context_survives(cuda_device):
    """A peer that never arrives: the bounded wait gives up, records ERR_PEER_WAIT (4), and the
    CUDA context stays usable.  Both "ranks'" signal pads are local memory of this GPU."""
    from maloq_b200.ops import kernels

    lib = kernels.lib()
    kernels.error_status(True)
    pads = torch.zeros(2, 8, dtype=torch.int32, device=cuda_device)
    ptrs = torch.tensor([pads[0].data_ptr(), pads[1].data_ptr()], dtype=torch.int64, device=cuda_device)
    lib.peer_barrier(ptrs.data_ptr(), 0, 2, 1, 0, 2000)  # rank 0 of 2; rank 1 never signals
    torch.cuda.synchronize()
    assert kernels.error_status(True) == 4
    assert pads[1, 0].item() == 1  # rank 0 did signal its peer slot
    assert torch.ones(3, device=cuda_device).sum().item() == 3
    assert kernels.error_status() == 0


def test_masked_peer_barrier_waits_only_for_members(cuda_device):
    """A member mask limits the barrier to halo neighbours: with only this rank in the mask
    (rank 0 of 3) nothing is waited for and nothing is signalled to the others; with rank 2 in
    the mask and rank 2 silent, the bounded wait runs out and records ERR_PEER_WAIT.  All three
    "ranks'" pads are local memory of this GPU."""
    from maloq_b200.ops import kernels

    lib = kernels.lib()
    kernels.error_status(True)
    pads = torch.zeros(3, 8, dtype=torch.int32, device=cuda_device)
    ptrs = torch.tensor([pads[i].data_ptr() for i in range(3)], dtype=torch.int64, device=cuda_device)
    lib.peer_barrier_mask(ptrs.data_ptr(), 0, 3, 1, 0, 2000, 0b001)
    torch.cuda.synchronize()
    assert kernels.error_status(True) == 0
    assert pads[1, 0].item() == 0 and pads[2, 0].item() == 0 and pads[0, 0].item() == 1
    lib.peer_barrier_mask(ptrs.data_ptr(), 0, 3, 2, 0, 2000, 0b101)
    torch.cuda.synchronize()
    assert kernels.error_status(True) == 4
    assert pads[2, 0].item() == 2 and pads[1, 0].item() == 0  # signalled the member only
    assert kernels.error_status() == 0


def test_peer_barrier_rejects_a_stale_epoch(cuda_device):
    """A peer whose flag still holds an older epoch has not arrived: the wait for epoch 6 runs
    out while the peer shows 5; once the peer shows 6 (or a later epoch) the barrier passes."""
    from maloq_b200.ops import kernels

    lib = kernels.lib()
    kernels.error_status(True)
    pads = torch.zeros(2, 8, dtype=torch.int32, device=cuda_device)
    ptrs = torch.tensor([pads[0].data_ptr(), pads[1].data_ptr()], dtype=torch.int64, device=cuda_device)
    pads[0, 1] = 5  # rank 1's flag in rank 0's pad: a previous step's epoch
    lib.peer_barrier(ptrs.data_ptr(), 0, 2, 6, 0, 2000)
    torch.cuda.synchronize()
    assert kernels.error_status(True) == 4
    pads[0, 1] = 7
    lib.peer_barrier(ptrs.data_ptr(), 0, 2, 6, 0, 2000)
    torch.cuda.synchronize()
    assert kernels.error_status(True) == 0


def test_peer_timeout_raises_comm_timeout_on_the_host(cuda_device):
    """The host-side status check turns the recorded peer timeout into CommTimeoutError (what
    the trainer raises after a step) and clears the word."""
    import pytest

    from maloq_b200.ops import kernels
    from maloq_b200.train.trainer import SplitTrainer

    lib = kernels.lib()
    kernels.error_status(True)
    pads = torch.zeros(2, 8, dtype=torch.int32, device=cuda_device)
    ptrs = torch.tensor([pads[0].data_ptr(), pads[1].data_ptr()], dtype=torch.int64, device=cuda_device)
    lib.peer_barrier(ptrs.data_ptr(), 0, 2, 1, 0, 2000)
    with pytest.raises(kernels.CommTimeoutError):
        SplitTrainer.check_status("test step")
    kernels.check_device_status()  # cleared: no raise


def test_edge_rotation_rows_orthonormal_and_empty(cuda_device):
    """The m-truncated rows of D are orthonormal (rot rot^T = 1), and zero edges is a no-op."""
    from maloq_b200.core import sph
    from maloq_b200.models.so3 import CoefficientMapping
    from maloq_b200.ops import misc_native

    mp = CoefficientMapping(6, 2).to(cuda_device)
    Js = [j.to(cuda_device) for j in sph.J_matrices(6)]
    v = torch.randn(777, 3, device=cuda_device)
    rot = misc_native.edge_rotation(v, 6, 2, Js, mp)
    eye = torch.eye(rot.shape[1], device=cuda_device).expand(rot.shape[0], -1, -1)
    assert (rot @ rot.transpose(1, 2) - eye).abs().max().item() < 1e-5
    empty = misc_native.edge_rotation(v[:0], 6, 2, Js, mp)
    assert empty.shape == (0, rot.shape[1], rot.shape[2])


def test_edge_inputs_kernel_and_gradients(cuda_device):
    """Radial-MLP input rows in one kernel (bf16) vs embedding lookups + Gaussian expansion +
    concatenation in fp32; the embedding-table gradients (one-hot GEMMs) vs autograd."""
    from maloq_b200.ops import misc_native

    torch.manual_seed(0)
    E, V, C, NB = 5000, 100, 128, 128
    src_z = torch.randint(1, 20, (E,), device=cuda_device)
    dst_z = torch.randint(1, 20, (E,), device=cuda_device)
    attr = torch.rand(E, 4, device=cuda_device) * 6
    sw = torch.randn(V, C, device=cuda_device, requires_grad=True)
    dw = torch.randn(V, C, device=cuda_device, requires_grad=True)
    off = torch.linspace(0, 6, NB, device=cuda_device)
    coeff = -0.5 / float(off[1] - off[0]) ** 2
    out = misc_native.edge_inputs(src_z, dst_z, attr, sw, dw, off, coeff)
    ref = torch.cat([sw[src_z], torch.exp(coeff * (attr[:, :1] - off.view(1, -1)) ** 2), dw[dst_z]], 1)
    assert out.dtype == torch.bfloat16
    assert ((out.float() - ref).abs() <= 2 ** -8 * ref.abs() + 1e-30).all()
    g = torch.randn_like(ref)
    ga = torch.autograd.grad((out.float() * g).sum(), [sw, dw])
    gr = torch.autograd.grad((ref * g).sum(), [sw, dw])
    for a, b in zip(ga, gr):
        assert ((a - b).norm() / b.norm()).item() < 1e-2
    from maloq_b200.ops import kernels

    assert kernels.error_status() == 0


@pytest.mark.parametrize("M,N,dtype,col0", [(1, 3, torch.bfloat16, 0), (300, 40, torch.float32, 8),
                                            (45948, 128, torch.bfloat16, 128), (151553, 8, torch.float32, 0),
                                            (20000, 3072, torch.bfloat16, 0)])
def test_colsum_matches_fp32_sum(cuda_device, M, N, dtype, col0):
    """Column sums of a row-strided slice against a PyTorch fp32 sum; repeated calls give the same bits."""
    from maloq_b200.ops import kernels

    torch.manual_seed(M)
    full = torch.randn(M, N + col0 + 8, device=cuda_device).to(dtype)
    X = full[:, col0:col0 + N]
    out = kernels.colsum(X)
    ref = X.double().sum(0)
    assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-4 * max(1.0, M ** 0.5))
    assert torch.equal(out, kernels.colsum(X))
    assert kernels.error_status() == 0


def test_weight_pack_and_segment_sums(cuda_device):
    """bf16 weight operand copies, pair matrices and pair-matrix gradients (one call, more jobs
    than one launch takes) and row-segment sums against their PyTorch definitions."""
    from maloq_b200.ops import kernels
    from maloq_b200.ops import weights as W

    torch.manual_seed(1)
    srcs, dsts, kinds, refs = [], [], [], []
    for i in range(60):
        kind = i % 5
        h, k = 8 + i % 7, 16 + (3 * i) % 11
        S = torch.randn(*((3, 2 * h, k) if kind == 1 and i % 2 else (2 * h, 2 * k) if kind == 4 else (2 * h, k)),
                        device=cuda_device)
        ref = [lambda: S, lambda: S.transpose(-1, -2), lambda: W._pair(S), lambda: W._pair(S).t(),
               lambda: W.pair_grad(S)][kind]()
        refs.append(ref.contiguous() if kind == 4 else ref.to(torch.bfloat16).contiguous())
        dsts.append(torch.empty_like(refs[-1]))
        srcs.append(S)
        kinds.append(kind)
    kernels.lib().weight_pack(srcs, dsts, kinds)
    for d, r, kd in zip(dsts, refs, kinds):
        assert torch.allclose(d, r, rtol=1e-6, atol=1e-6) if kd == 4 else torch.equal(d, r)
    X = torch.randn(5 * 16 * 25, 128 * 128 // 4, device=cuda_device)
    seg = [l * l * 16 for l in range(6)]
    out = torch.empty(5, X.shape[1], device=cuda_device)
    kernels.lib().colsum_segments(X, seg, out)
    ref = torch.stack([X[a:b].double().sum(0) for a, b in zip(seg[:-1], seg[1:])])
    assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-3)
    assert kernels.error_status() == 0
