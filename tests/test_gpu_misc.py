"""usaf_dot (the per-step scalar readback): against a float64 torch reference
(relative error <= 1e-5, fp32 accumulation), reproducible bit-for-bit across
calls, for aligned (16-byte vector) and unaligned inputs, fp32 and bf16."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


@pytest.mark.parametrize("n", [0, 1, 17, 4099, 8 * 1024 * 1024 + 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("offset", [0, 1])
def test_dot(dev, n, dtype, offset):
    from usaf_b200 import _lib
    g = torch.Generator(device=dev).manual_seed(n + offset)
    a = torch.randn(n + offset, device=dev, generator=g).to(dtype)[offset:]
    b = torch.randn(n + offset, device=dev, generator=g).to(dtype)[offset:]
    out = torch.full((2,), float("nan"), device=dev)
    for i in range(2):
        _lib.call("usaf_dot", _lib.ptr(a), _lib.ptr(b), _lib.dtype_code(dtype), n, _lib.ptr(out[i:]),
                  _lib.stream())
    torch.cuda.synchronize()
    ref = (a.double() * b.double()).sum().item()
    assert out[0].item() == out[1].item()
    scale = (a.double().abs() * b.double().abs()).sum().item()
    assert abs(out[0].item() - ref) <= 1e-5 * max(scale, 1e-30) + 1e-6
