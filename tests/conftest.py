import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")
    config.addinivalue_line("markers", "slow: long-running (full-size configs)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("needs an sm_100 device")
    return True


def spawn_ranks(fn, args, nprocs, seconds):
    """Run fn(rank, *args) in nprocs spawned processes; fail (and kill those
    processes, by PID) if they have not all finished within ``seconds``."""
    import time
    import torch.multiprocessing as mp
    ctx = mp.start_processes(fn, args=args, nprocs=nprocs, join=False, start_method="spawn")
    deadline = time.monotonic() + seconds
    while not ctx.join(timeout=2):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            for p in ctx.processes:
                p.join(10)
            pytest.fail(f"ranks did not finish within {seconds} s")
