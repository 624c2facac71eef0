"""Host transfers and zero-copy exchange (CPU paths here; the pinned copy runs on the GPU)."""
import numpy as np
import pytest
import torch

from flare_b200.utils.transfer import from_external, to_external, to_host


def test_dlpack_views_share_memory():
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    t = from_external(a)
    t[0, 0] = 42.0
    assert a[0, 0] == 42.0  # zero copy
    b = np.from_dlpack(t)
    b[2, 3] = -1.0
    assert float(t[2, 3]) == -1.0
    u = torch.from_dlpack(to_external(t))
    assert u.data_ptr() == t.data_ptr()


def test_to_host_on_cpu_returns_the_tensor():
    t = torch.arange(5)
    h = to_host(t)
    assert h.ready() and torch.equal(h.result(), t)


@pytest.mark.gpu
def test_to_host_pinned_copy_on_the_stream(cuda):
    x = torch.arange(1 << 20, device=cuda, dtype=torch.float32)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y = x * 2
    h = to_host(y, stream=s)
    assert h.tensor.is_pinned()
    out = h.result()
    assert torch.equal(out, (x * 2).cpu())
    h2 = to_host(y, stream=s)  # the released pinned buffer is reused
    assert torch.equal(h2.result(), out)
