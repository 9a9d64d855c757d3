import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "flash-attention-rdna2_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(autouse=True, scope="module")
def _device_error_flags_clear(request):
    """Every GPU test module must end with no device-side error recorded (a pipeline wait that
    gave up, a bad page index, a rotary position past its table): such a kernel returns wrong
    values without a host error, so the flag is read here after the module's tests."""
    import torch
    gpu_module = any("gpu" in it.keywords for it in request.session.items
                     if it.module is request.module) if hasattr(request, "module") else False
    if not (gpu_module and torch.cuda.is_available()):
        yield
        return
    import fable_attn
    fable_attn.device_error(clear=True)
    yield
    flags = fable_attn.device_error(clear=True)
    assert flags == 0, f"device error bits 0x{flags:x} recorded during {request.module.__name__}"
