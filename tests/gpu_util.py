"""Helpers for the GPU parity tests: torch is used only to hold device memory
and the current stream; every computation under test goes through the C ABI."""
import ctypes

import numpy as np


def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError('GPU tests need a CUDA device (run them with -m gpu on a B200)')
    return torch


def dev(a):
    torch = torch_cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


class Keep:
    """Holds every device tensor made through it until the test ends: a bare
    data_ptr() of a temporary would point into freed (and reused) memory."""

    def __init__(self):
        self.tensors = []

    def __call__(self, a):
        t = dev(a)
        self.tensors.append(t)
        return vp(t)


def vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    torch = torch_cuda()
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def sync():
    torch_cuda().cuda.synchronize()


def bf16_round(a):
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7fff + ((u >> 16) & 1)) & 0xffff0000
    return u.astype(np.uint32).view(np.float32)


def to_bits(a):
    a = np.ascontiguousarray(a, np.float32)
    bits = a.view(np.uint32)
    assert not (bits & 0xffff).any()
    return (bits >> 16).astype(np.uint16)


def from_bits(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def ulp_bf16(x):
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    x = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.maximum(x, 1e-30)))
    return np.exp2(e - 7)


def assert_bf16_close(got, exp, min_equal=0.99, max_ulps=1.0, what='', mag=None):
    """Bound for bf16 outputs whose fp32 pre-rounding values differ only by
    summation order: nearly all equal, the rest within max_ulps bf16 ulps.
    `mag` (optional, same shape) is an intermediate whose ulp also counts, e.g.
    the linear term of a residual sum that can cancel against the residual."""
    got = np.asarray(got, np.float32).ravel()
    exp = np.asarray(exp, np.float32).ravel()
    assert got.shape == exp.shape, what
    assert np.isfinite(got).all(), what
    eq = (got == exp).mean()
    diff = np.abs(got.astype(np.float64) - exp)
    # plus a floor at 2^-12 of the tensor's scale for outputs that are sums
    # with cancellation (tiny results whose own ulp is below fp32 noise)
    ref_mag = np.maximum(np.abs(got), np.abs(exp))
    if mag is not None:
        ref_mag = np.maximum(ref_mag, np.abs(np.asarray(mag, np.float32).ravel()))
    bound = max_ulps * ulp_bf16(ref_mag) + 2.0 ** -12 * float(np.abs(exp).max()) + 1e-30
    worst = float((diff / bound).max())
    assert eq >= min_equal, f'{what}: only {eq:.4f} bit-equal'
    assert worst <= 1.0, f'{what}: max difference {worst:.2f} x {max_ulps} ulp'
    return eq
