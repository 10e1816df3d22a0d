"""Index-checked build (MALOQ_BOUNDS_CHECK=1): out-of-range data indices are reported as
error 5 / BoundsError and the access is skipped.  Each case runs in a fresh process that
loads the checked library.  The bad index points one row past a view of a larger buffer, so
the memory it names exists even for a kernel that did not check."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASE = textwrap.dedent("""
    import sys, torch
    sys.path.insert(0, {root!r})
    from maloq_b200.ops import kernels
    lib = kernels.lib()
    assert lib.bounds_checked(), "checked build not loaded"
    dev = torch.device("cuda", 0)
    E, N, C, S, R, Cin = 64, 10, 128, 25, 19, 256
    store = torch.randn(N + 4, S, C, device=dev)
    X = store[:N]                       # N valid rows; row N exists physically
    src = torch.randint(0, N, (E,), device=dev)
    dst = torch.sort(torch.randint(0, N, (E,), device=dev)).values
    rot = torch.randn(E, R, S, device=dev)
    rad = torch.randn(E, 12 * Cin, device=dev).bfloat16()
    A0 = torch.zeros(E, R * Cin, device=dev, dtype=torch.bfloat16)
    lib.gather_rotate_fwd(4, 2, X, None, src, dst, rot, rad, A0, Cin, 0, None, None, 0)
    torch.cuda.synchronize()
    assert kernels.error_status(True) == 0
    bad = src.clone(); bad[5] = N       # one past the last valid row
    A1 = torch.zeros_like(A0)
    lib.gather_rotate_fwd(4, 2, X, None, bad, dst, rot, rad, A1, Cin, 0, None, None, 0)
    try:
        kernels.check_device_status("gather")
        raise SystemExit("no error recorded")
    except kernels.BoundsError:
        pass
    assert torch.equal(A1[5], torch.zeros_like(A1[5])), "out-of-range edge was not skipped"
    keep = torch.arange(E, device=dev) != 5
    assert torch.equal(A1[keep], A0[keep]), "in-range edges changed"
    print("OK")
""")


def test_checked_build_reports_and_skips_out_of_range_gather_source(cuda_device):
    env = dict(os.environ, MALOQ_BOUNDS_CHECK="1")
    r = subprocess.run([sys.executable, "-c", CASE.format(root=ROOT)], capture_output=True, text=True, env=env,
                       timeout=900)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


def test_default_build_is_unchecked():
    from maloq_b200.ops import kernels

    assert not kernels.lib().bounds_checked()
