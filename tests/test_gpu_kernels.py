"""The kernel ABI (mgc_cuda_gemm, _conv_nhwc, _softmax, _layer_norm, _pool_nhwc, _depthwise_nhwc,
_reduce_mid) against a plain PyTorch fp32 reference of the same operation and, where it is
built, the reference's own C kernels (oracle/_ref/libmgc_ref_kernels.so, mgc_kernels.c)."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from mgc_cuda.runtime import library, last_error

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libmgc_ref_kernels.so"


def dev(a: np.ndarray) -> "torch.Tensor":
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t: "torch.Tensor | None") -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ok(st: int) -> None:
    assert st == 0, last_error()


def ref_lib() -> ctypes.CDLL | None:
    return ctypes.CDLL(str(REF_LIB)) if REF_LIB.exists() else None


def tf32_round(a: np.ndarray) -> np.ndarray:
    """fp32 rounded to the nearest TF32 value (10 mantissa bits, ties away from zero): what a
    TFLOAT32 tensor map does to an operand on load."""
    from mgc_cuda.lowering import tf32_split

    return tf32_split(a)[0]


@pytest.mark.parametrize("kmajor", [False, True])
@pytest.mark.parametrize("precision", [0, 1, 2])
@pytest.mark.parametrize("m,n,k,act", [(1, 1000, 2048, 0), (197, 77, 129, 1), (512, 256, 64, 3), (64, 3072, 768, 4),
                                       (300, 200, 100, 1)])
def test_gemm_vs_torch(m: int, n: int, k: int, act: int, precision: int, kmajor: bool) -> None:
    """The kernel ABI's GEMM does the arithmetic its precision names, or refuses:
    * fp32 (0): exact fp32 on the CUDA cores, any layout, within 1e-5 of a float64 product;
    * tf32 (1): the tcgen05 tensor cores when A and B are K-major with aligned rows (K and N
      multiples of 4), matching a float64 product of the TF32-rounded operands within 1e-4 of the
      output scale (fp32 accumulation); any other layout returns MGC_CUDA_UNSUPPORTED and leaves
      the output untouched;
    * 3xtf32 (2): MGC_CUDA_UNSUPPORTED (the strict split needs weights prepared at load time)."""
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32) * 0.05
    bias = rng.standard_normal(n).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    A, Bi, R = dev(a), dev(bias), dev(res)
    B = dev(np.ascontiguousarray(b.T)) if kmajor else dev(b)
    b_rs, b_cs = (1, k) if kmajor else (n, 1)
    C = torch.full((m, n), float("nan"), device="cuda")
    lib = library()
    st = lib.mgc_cuda_gemm(m, n, k, 1, ptr(A), k, 1, 0, ptr(B), b_rs, b_cs, 0, ptr(C), n, 0, 1.0, ptr(Bi), 1, ptr(R), n,
                           0, 1.0, act, 0.0, 6.0, precision, stream())
    torch.cuda.synchronize()
    supported = precision == 0 or (precision == 1 and kmajor and k % 4 == 0 and n % 4 == 0)
    if not supported:
        assert st == 3, (st, last_error())
        assert "MGC_PREC_FP32" in last_error()
        assert bool(torch.isnan(C).all())
        return
    ok(st)
    if precision == 1:
        a, b = tf32_round(a), tf32_round(b)
    y = a.astype(np.float64) @ b.astype(np.float64) + bias + res
    y = torch.from_numpy(y)
    y = {0: y, 1: torch.relu(y), 3: torch.nn.functional.gelu(y), 4: torch.nn.functional.gelu(y, approximate="tanh")}[act]
    err = float((C.double().cpu() - y).abs().max())
    scale = float(y.abs().max())
    tol = 1e-4 if precision == 1 else 1e-5
    assert err <= tol * max(scale, 1.0), f"err {err:.3g} scale {scale:.3g}"


def test_gemm_tf32_batched_dynamic_b() -> None:
    """TF32 batched product of two activations (attention's form) through the kernel ABI: one
    batch dimension with a constant stride, on the tensor cores."""
    rng = np.random.default_rng(11)
    batch, m, n, k = 6, 128, 128, 64
    a = rng.standard_normal((batch, m, k)).astype(np.float32)
    bt = rng.standard_normal((batch, n, k)).astype(np.float32)  # K-major B
    A, B = dev(a), dev(bt)
    C = torch.empty((batch, m, n), device="cuda")
    ok(library().mgc_cuda_gemm(m, n, k, batch, ptr(A), k, 1, m * k, ptr(B), 1, k, n * k, ptr(C), n, m * n, 1.0, None, 0,
                               None, 0, 0, 1.0, 0, 0.0, 6.0, 1, stream()))
    torch.cuda.synchronize()
    want = np.einsum("bmk,bnk->bmn", tf32_round(a).astype(np.float64), tf32_round(bt).astype(np.float64))
    err = float(np.abs(C.cpu().numpy() - want).max())
    assert err <= 1e-4 * float(np.abs(want).max())


@pytest.mark.parametrize("shape", [(2, 14, 14, 64, 3, 1, 1), (1, 56, 56, 64, 1, 1, 0), (2, 28, 28, 32, 3, 2, 1), (1, 32, 32, 3, 7, 2, 3)])
def test_conv_nhwc_vs_torch(shape: tuple) -> None:
    """Exact fp32 (precision 0) against a float64 convolution; TF32 and 3xTF32 are refused with
    MGC_CUDA_UNSUPPORTED (their tensor-core forms read weights the lowering lays out K-major)."""
    n, h, w, c, kk, s, p = shape
    co = 48
    rng = np.random.default_rng(h * c)
    x = rng.standard_normal((n, h, w, c)).astype(np.float32)
    wt = (rng.standard_normal((kk, kk, c, co)) * 0.1).astype(np.float32)
    bias = rng.standard_normal(co).astype(np.float32)
    oh = (h + 2 * p - kk) // s + 1
    ow = (w + 2 * p - kk) // s + 1
    X, W, Bi = dev(x), dev(wt), dev(bias)
    Y = torch.empty((n, oh, ow, co), device="cuda")
    lib = library()
    for precision in (1, 2):
        st = lib.mgc_cuda_conv_nhwc(n, h, w, c, kk, kk, s, s, 1, 1, p, p, oh, ow, co, ptr(X), ptr(W), ptr(Bi), None,
                                    1, 0.0, 6.0, ptr(Y), precision, stream())
        assert st == 3 and "MGC_PREC_FP32" in last_error()
    ok(lib.mgc_cuda_conv_nhwc(n, h, w, c, kk, kk, s, s, 1, 1, p, p, oh, ow, co, ptr(X), ptr(W), ptr(Bi), None,
                              1, 0.0, 6.0, ptr(Y), 0, stream()))
    torch.cuda.synchronize()
    ref = torch.nn.functional.conv2d(X.permute(0, 3, 1, 2).double(), W.permute(3, 2, 0, 1).double(), Bi.double(),
                                     stride=s, padding=p).relu().permute(0, 2, 3, 1)
    err = float((Y.double() - ref).abs().max())
    assert err <= 1e-5 * max(float(ref.abs().max()), 1.0)


def test_softmax_layer_norm_reduce_vs_torch_and_reference_c() -> None:
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((48, 128)) * 4).astype(np.float32)
    X = dev(x)
    Y = torch.empty_like(X)
    lib = library()
    ok(lib.mgc_cuda_softmax(48, 128, 1, ptr(X), ptr(Y), 0, stream()))
    torch.cuda.synchronize()
    np.testing.assert_allclose(Y.cpu().numpy(), torch.softmax(X.double(), -1).cpu().numpy(), rtol=1e-5, atol=1e-7)
    g = (rng.random(128) + 0.5).astype(np.float32)
    b = rng.standard_normal(128).astype(np.float32)
    G, B = dev(g), dev(b)
    ok(lib.mgc_cuda_layer_norm(48, 128, ptr(X), ptr(G), ptr(B), 1e-5, ptr(Y), stream()))
    torch.cuda.synchronize()
    ln = torch.nn.functional.layer_norm(X.double(), (128,), G.double(), B.double(), 1e-5)
    np.testing.assert_allclose(Y.cpu().numpy(), ln.cpu().numpy(), rtol=1e-5, atol=2e-5)
    R = torch.empty((48,), device="cuda")
    ok(lib.mgc_cuda_reduce_mid(0, 48, 128, 1, ptr(X), ptr(R), stream()))
    torch.cuda.synchronize()
    np.testing.assert_allclose(R.cpu().numpy(), x.astype(np.float64).mean(axis=1), rtol=1e-5, atol=1e-6)
    ref = ref_lib()
    if ref is not None:  # the reference's own C kernels, same inputs
        out = np.empty_like(x)
        ref.mgc_layer_norm.argtypes = [ctypes.c_long, ctypes.c_long] + [ctypes.c_void_p] * 3 + [ctypes.c_float, ctypes.c_void_p]
        ref.mgc_layer_norm(48, 128, x.ctypes.data, g.ctypes.data, b.ctypes.data, 1e-5, out.ctypes.data)
        ok(lib.mgc_cuda_layer_norm(48, 128, ptr(X), ptr(G), ptr(B), 1e-5, ptr(Y), stream()))
        torch.cuda.synchronize()
        np.testing.assert_allclose(Y.cpu().numpy(), out, rtol=1e-5, atol=2e-5)


def test_pool_and_depthwise_vs_torch() -> None:
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 17, 17, 32)).astype(np.float32)
    X = dev(x)
    Y = torch.empty((2, 9, 9, 32), device="cuda")
    lib = library()
    ok(lib.mgc_cuda_pool_nhwc(1, 2, 17, 17, 32, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 9, 9, 0, ptr(X), ptr(Y), stream()))
    torch.cuda.synchronize()
    ref = torch.nn.functional.max_pool2d(X.permute(0, 3, 1, 2), 3, 2, 1).permute(0, 2, 3, 1)
    np.testing.assert_array_equal(Y.cpu().numpy(), ref.cpu().numpy())
    w = (rng.standard_normal((3, 3, 32)) * 0.3).astype(np.float32)
    b = rng.standard_normal(32).astype(np.float32)
    W, B = dev(w), dev(b)
    ok(lib.mgc_cuda_depthwise_nhwc(2, 17, 17, 32, 3, 3, 2, 2, 1, 1, 1, 1, 9, 9, ptr(X), ptr(W), ptr(B), None, 2,
                                   0.0, 6.0, ptr(Y), stream()))
    torch.cuda.synchronize()
    ref = torch.nn.functional.conv2d(X.permute(0, 3, 1, 2).double(), W.permute(2, 0, 1).unsqueeze(1).double(),
                                     B.double(), stride=2, padding=1, groups=32).clamp(0, 6).permute(0, 2, 3, 1)
    np.testing.assert_allclose(Y.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n,h,w,c,s,pad,act,res", [
    (2, 14, 14, 384, 1, 1, 2, False),  # MobileNetV2's 14 x 14 layers: four channels per thread
    (3, 7, 7, 960, 1, 1, 2, True),      # 7 x 7, 30 channel vectors per block, residual
    (2, 15, 9, 18, 2, 1, 1, True),      # C % 4 == 2: two channels per thread, odd sizes
    (1, 20, 33, 6, 1, 0, 0, False),     # no padding, two channels per thread
    (2, 28, 28, 144, 2, 1, 2, False),   # stride 2, even input
    (1, 5, 4, 40, 2, 0, 1, True),       # one output row and column per band
    (4, 112, 112, 32, 1, 1, 2, False),  # MobileNetV2's first depthwise layer
    (130, 7, 7, 960, 1, 1, 2, True),    # more blocks than one wave, residual
    (300, 8, 8, 512, 2, 1, 1, False),   # more blocks than one wave at stride 2
])
def test_depthwise_bands_vs_torch(n: int, h: int, w: int, c: int, s: int, pad: int, act: int, res: bool) -> None:
    """The row-band depthwise forms (3x3, stride 1 or 2; a shared-memory ring of input rows
    filled by TMA, or by cp.async with four or two channels per thread; any padding) against a
    float64 depthwise convolution, and bit-identical to each other (the same order of
    accumulation); the older forms (MGC_CUDA_DW=legacy) give the same values to the same
    tolerance."""
    import os

    rng = np.random.default_rng(h * w * c + s)
    oh, ow = (h + 2 * pad - 3) // s + 1, (w + 2 * pad - 3) // s + 1
    x = rng.standard_normal((n, h, w, c)).astype(np.float32)
    wt = (rng.standard_normal((3, 3, c)) * 0.3).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    r = rng.standard_normal((n, oh, ow, c)).astype(np.float32)
    X, W, B, R = dev(x), dev(wt), dev(b), dev(r)
    ref = torch.nn.functional.conv2d(X.permute(0, 3, 1, 2).double(), W.permute(2, 0, 1).unsqueeze(1).double(),
                                     B.double(), stride=s, padding=pad, groups=c).permute(0, 2, 3, 1)
    if res:
        ref = ref + R.double()
    ref = {0: ref, 1: ref.relu(), 2: ref.clamp(0, 6)}[act]
    outs = []
    forms = ("tma", "ring", "ring2", "legacy")
    for form in forms:
        os.environ["MGC_CUDA_DW"] = form
        try:
            Y = torch.full((n, oh, ow, c), float("nan"), device="cuda")
            ok(library().mgc_cuda_depthwise_nhwc(n, h, w, c, 3, 3, s, s, 1, 1, pad, pad, oh, ow, ptr(X), ptr(W),
                                                 ptr(B), ptr(R) if res else None, act, 0.0, 6.0, ptr(Y), stream()))
            torch.cuda.synchronize()
        finally:
            del os.environ["MGC_CUDA_DW"]
        np.testing.assert_allclose(Y.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-5, err_msg=f"form {form}")
        outs.append(Y.cpu().numpy())
    for form, out in zip(forms[1:-1], outs[1:-1]):
        np.testing.assert_array_equal(out, outs[0], err_msg=form)


@pytest.mark.parametrize("n,h,w,c,s,act", [(2, 30, 45, 48, 1, 2), (1, 57, 33, 64, 2, 1), (3, 19, 70, 32, 1, 0),
                                           (2, 40, 36, 16, 2, 2)])
def test_depthwise_tiles_vs_torch(n: int, h: int, w: int, c: int, s: int, act: int) -> None:
    """The shared-memory tiled depthwise form (3x3, stride 1 or 2, 16 or more output columns;
    channel chunks of 32 or 16) against a float64 depthwise convolution, with a residual and
    ReLU / Clip; sizes that leave partial row, column and channel tiles."""
    rng = np.random.default_rng(h * w + c)
    oh, ow = (h + 2 - 3) // s + 1, (w + 2 - 3) // s + 1
    x = rng.standard_normal((n, h, w, c)).astype(np.float32)
    wt = (rng.standard_normal((3, 3, c)) * 0.3).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    r = rng.standard_normal((n, oh, ow, c)).astype(np.float32)
    X, W, B, R = dev(x), dev(wt), dev(b), dev(r)
    Y = torch.full((n, oh, ow, c), float("nan"), device="cuda")
    ok(library().mgc_cuda_depthwise_nhwc(n, h, w, c, 3, 3, s, s, 1, 1, 1, 1, oh, ow, ptr(X), ptr(W), ptr(B), ptr(R), act,
                                         0.0, 6.0, ptr(Y), stream()))
    torch.cuda.synchronize()
    ref = torch.nn.functional.conv2d(X.permute(0, 3, 1, 2).double(), W.permute(2, 0, 1).unsqueeze(1).double(),
                                     B.double(), stride=s, padding=1, groups=c).permute(0, 2, 3, 1) + R.double()
    ref = {0: ref, 1: ref.relu(), 2: ref.clamp(0, 6)}[act]
    np.testing.assert_allclose(Y.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-5)
