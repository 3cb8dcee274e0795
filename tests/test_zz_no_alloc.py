"""mgc_cuda_conv_nhwc_noalloc: the convolution entry point for callers that cannot allocate
device memory (code that plans all of its memory up front and never allocates afterwards, or
that runs where cudaMalloc is not allowed). Its im2col scratch is a fixed 16 MiB device array
inside the library instead of a buffer it allocates, so the only memory it touches is the
caller's inputs and outputs plus that array.

The test calls it twice in a row through the C ABI, with different shapes, and checks each
result against the existing mgc_cuda_conv_nhwc on the same inputs and against a float64
convolution (exact-fp32 arithmetic, compared at the kernel tests' 1e-5 relative tolerance). It
checks the property that defines it: after a first call, further calls leave the device's free
memory unchanged (nothing allocated, nothing freed). It also checks that a patch matrix larger
than the array is refused with a clear error. The file is named to be collected last, so a run
that stops at the first failure has run every other test first; it passes alone in a fresh
process as well."""

from __future__ import annotations

import numpy as np
import pytest

from mgc_cuda.runtime import library, last_error

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024


def _conv_args(n: int, h: int, w: int, c: int, k: int, s: int, p: int, co: int, seed: int):
    rng = np.random.default_rng(seed)
    oh = (h + 2 * p - k) // s + 1
    ow = (w + 2 * p - k) // s + 1
    x = torch.from_numpy(rng.standard_normal((n, h, w, c)).astype(np.float32)).cuda()
    wt = torch.from_numpy((rng.standard_normal((k, k, c, co)) * 0.2).astype(np.float32)).cuda()
    bias = torch.from_numpy(rng.standard_normal(co).astype(np.float32)).cuda()
    res = torch.from_numpy(rng.standard_normal((n, oh, ow, co)).astype(np.float32)).cuda()
    return (n, h, w, c, k, k, s, s, 1, 1, p, p, oh, ow, co), x, wt, bias, res


def _run(fn_name: str, geo, x, wt, bias, res, act: int, free: list[int] | None = None) -> "torch.Tensor":
    """One call through the C ABI; with `free`, the device's free bytes just before and just after
    the call (the output buffer is allocated before the first reading) are appended to it."""
    lib = library()
    n, oh, ow, co = geo[0], geo[12], geo[13], geo[14]
    y = torch.full((n, oh, ow, co), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    if free is not None:
        free.append(torch.cuda.mem_get_info()[0])
    fn = getattr(lib, fn_name)
    if fn_name == "mgc_cuda_conv_nhwc":
        st = fn(*geo, x.data_ptr(), wt.data_ptr(), bias.data_ptr(), res.data_ptr(), act, 0.0, 6.0, y.data_ptr(),
                0, stream)
    else:
        st = fn(*geo, x.data_ptr(), wt.data_ptr(), bias.data_ptr(), res.data_ptr(), act, 0.0, 6.0, y.data_ptr(),
                stream)
    assert st == 0, last_error()
    torch.cuda.synchronize()
    if free is not None:
        free.append(torch.cuda.mem_get_info()[0])
    return y


def _float64_conv(geo, x, wt, bias, res, act: int) -> "torch.Tensor":
    s, p = geo[6], geo[10]
    y = torch.nn.functional.conv2d(x.permute(0, 3, 1, 2).double(), wt.permute(3, 2, 0, 1).double(), bias.double(),
                                   stride=s, padding=p).permute(0, 2, 3, 1) + res.double()
    return y.relu() if act == 1 else y.clamp(0.0, 6.0)


def test_noalloc_conv_matches_the_allocating_entry_point_twice_in_a_row() -> None:
    # the stem shape of ResNet-50 (3 channels, 7x7 stride 2) and a 3x3 layer, one after the other
    free: list[int] = []
    for (n, h, w, c, k, s, p, co, act, seed) in ((1, 64, 64, 3, 7, 2, 3, 64, 1, 1), (2, 14, 14, 24, 3, 1, 1, 40, 2, 2)):
        geo, x, wt, bias, res = _conv_args(n, h, w, c, k, s, p, co, seed)
        want = _run("mgc_cuda_conv_nhwc", geo, x, wt, bias, res, act)
        got = _run("mgc_cuda_conv_nhwc_noalloc", geo, x, wt, bias, res, act, free)
        assert torch.isfinite(got).all()
        scale = max(float(want.abs().max()), 1.0)
        err = float((got.double() - want.double()).abs().max())
        assert err <= 1e-5 * scale, f"vs mgc_cuda_conv_nhwc: max abs err {err:.3g} (scale {scale:.3g})"
        err64 = float((got.double() - _float64_conv(geo, x, wt, bias, res, act)).abs().max())
        assert err64 <= 1e-5 * scale, f"vs float64: max abs err {err64:.3g} (scale {scale:.3g})"
    # the first call of the process may load the module's device code; every later call allocates
    # and frees nothing, so the free device memory around it does not move
    assert free[2] == free[3], f"the second call changed free device memory: {free}"
    geo, x, wt, bias, res = _conv_args(1, 64, 64, 3, 7, 2, 3, 64, 1)
    more: list[int] = []
    for _ in range(3):
        _run("mgc_cuda_conv_nhwc_noalloc", geo, x, wt, bias, res, 1, more)
    assert more[0::2] == more[1::2], f"repeated calls changed free device memory: {more}"


def test_noalloc_conv_refuses_a_patch_matrix_larger_than_its_scratch() -> None:
    # 2 x 112 x 112 output pixels x 147 patch floats (148 padded) is about 14.9 MB per image pair;
    # 4 images exceed the 16 MiB array
    geo, x, wt, bias, res = _conv_args(4, 224, 224, 3, 7, 2, 3, 8, 3)
    rows = geo[0] * geo[12] * geo[13]
    assert rows * 148 * 4 > NOALLOC_SCRATCH_BYTES
    lib = library()
    y = torch.empty((geo[0], geo[12], geo[13], geo[14]), device="cuda")
    st = lib.mgc_cuda_conv_nhwc_noalloc(*geo, x.data_ptr(), wt.data_ptr(), bias.data_ptr(), res.data_ptr(), 1, 0.0,
                                        6.0, y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 2
    assert "static scratch" in last_error()
