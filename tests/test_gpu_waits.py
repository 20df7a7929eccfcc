"""Failure detection of the kernels' bounded waits, on the GPU without a fault.

Every wait of the band kernels on a TMA bulk copy is bounded (1 s after its
first failed poll); a wait that gives up is counted process-wide
(``cqt_wait_timeouts``) and in the wait-status word of the call's workspace
(``cqt_workspace_waits``), and the kernel finishes.  Healthy calls leave the
word at zero.  The test hook ``cqt_debug_expire_waits`` arms the staging
barriers for 16 bytes that never arrive -- a completion that nothing
delivers -- so every wait runs out; the test, in a child process of its own,
checks that the host reads a nonzero status, that the debug mode of the
Python layer raises, and that the context stays usable (the next normal call
is exact).  Nothing faults or hangs.
"""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def test_healthy_calls_leave_the_status_at_zero(dev):
    from flash_cqt_b200.engine import Engine
    eng = Engine.from_params([3, 4, 2], [8, 16, 32], 44100, 65536, dev)
    x = torch.randn(3, 65536, device=dev)
    y = eng.synthesis(eng.analysis(x))
    eng.adj_synthesis(eng.adj_analysis(eng.analysis(y)))
    assert eng.wait_status() == 0


_CHILD = textwrap.dedent("""
    import os, sys
    sys.path.insert(0, {root!r})
    import torch
    from flash_cqt_b200 import _native
    from flash_cqt_b200.engine import Engine
    from oracle.cqt_oracle import snr_db
    dev = torch.device("cuda:0")
    eng = Engine.from_params([3, 4, 2], [8, 16, 32], 44100, 65536, dev)
    x = torch.randn(1, 65536, device=dev)
    good = eng.analysis(x)
    torch.cuda.synchronize()
    assert eng.wait_status() == 0
    before = _native.wait_timeouts()
    L = _native.lib()
    L.cqt_debug_expire_waits(1)
    eng.analysis(x)                        # every staging wait runs out
    torch.cuda.synchronize()
    n = eng.wait_status()
    assert n > 0, n
    assert _native.wait_timeouts() - before >= n
    os.environ["FLASH_CQT_B200_CHECK_WAITS"] = "1"
    try:
        eng._ops = None                    # the Python path, where the debug check lives
        eng.analysis(x)
        raise SystemExit("debug mode did not raise")
    except RuntimeError as e:
        assert "bounded wait" in str(e), e
    os.environ["FLASH_CQT_B200_CHECK_WAITS"] = "0"
    L.cqt_debug_expire_waits(0)
    again = eng.analysis(x)                # the context is still usable
    torch.cuda.synchronize()
    assert eng.wait_status() == 0
    assert snr_db(good.cpu().numpy(), again.cpu().numpy()) > 200
    print("ok", n)
""")


def test_expired_waits_are_reported_and_context_survives(dev):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _CHILD.format(root=root)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().startswith("ok")
