import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for path in (ROOT, ROOT / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def native():
    """The C-ABI binding, with the native libraries built (a no-op when up to date)."""
    from lightdelta_b200 import build

    build.build_all()
    from lightdelta_b200 import capi

    capi.lib()
    return capi


@pytest.fixture(scope="session")
def device(native):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"built for sm_100a, found sm_{major}{minor}"
    from lightdelta_b200 import ops  # noqa: F401

    return torch.device("cuda", 0)


def pytest_terminal_summary(terminalreporter):
    """Largest measured outlier rate of each kind of tolerance check run in this session."""
    try:
        from helpers import MEASURED
    except ImportError:
        return
    if not MEASURED:
        return
    worst = {}
    for kind, what, count, size, ulps in MEASURED:
        rate = count / size if size else 0.0
        best = worst.get(kind)
        if best is None or rate > best[0]:
            worst[kind] = (rate, count, size, what, max(ulps, best[4] if best else 0))
        else:
            worst[kind] = best[:4] + (max(ulps, best[4]),)
    terminalreporter.write_line("tolerance checks, largest outlier rate per kind (rate, count, elements, where, max ulps):")
    for kind, (rate, count, size, what, ulps) in sorted(worst.items()):
        terminalreporter.write_line(f"  {kind}: {rate:.2e} ({count} of {size}) at '{what}', max {ulps} ulps overall")
