"""The allocation-free weight-gradient GEMM entry point ``nt_wgrad_splitk_noalloc``.

The entry point has no counterpart in the reference.  It is a plain C symbol exported by the
``_C`` library and is called here through ctypes, the way a caller without PyTorch would call
it.  Each case is compared with the PyTorch binding of the same GEMM (which takes its split-K
workspace from the caching allocator) on two consecutive calls, so a second call that reads the
first call's leftovers in the shared scratch array would show up as a mismatch.  The file is
named to be collected last, so that it runs both after the other GPU tests and on its own.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from nexttransformer_b200.ops._ext import ext
    mod = ext()
    handle = ctypes.CDLL(mod.__file__)
    fn = handle.nt_wgrad_splitk_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                   ctypes.c_void_p]
    cap = handle.nt_wgrad_splitk_noalloc_scratch_bytes
    cap.restype = ctypes.c_size_t
    cap.argtypes = []
    return mod, fn, cap()


def call(fn, dy, x, out, *, accumulate, alpha=1.0):
    """out[N, K] (+)= alpha * dy^T x  with dy [T, N], x [T, K] (both bf16, row-major)."""
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0),
              dy.shape[1], x.shape[1], dy.shape[0], alpha, int(accumulate), stream)


def reference(mod, dy, x, out, *, accumulate, alpha=1.0):
    mod.gemm(dy, True, x, True, out, mod.EPI_F32_ACC if accumulate else mod.EPI_F32, None, None, float(alpha),
             1.0, None)


# (tokens, out features, in features): the first two split the reduction (few output tiles),
# the third has enough tiles to run without scratch.
SHAPES = [(65536, 1280, 1280), (16384, 5120, 1280), (2048, 4096, 4096)]


@pytest.mark.parametrize("T,N,K", SHAPES)
@pytest.mark.parametrize("accumulate", [False, True])
def test_matches_allocating_entry_point(lib, T, N, K, accumulate):
    mod, fn, _ = lib
    g = torch.Generator(device="cuda").manual_seed(T + N + K)
    for trial in range(2):
        dy = torch.randn(T, N, device="cuda", generator=g).to(torch.bfloat16)
        x = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
        init = torch.randn(N, K, device="cuda", generator=g)
        ours, ref = init.clone(), init.clone()
        assert call(fn, dy, x, ours, accumulate=accumulate, alpha=0.5) == 0
        reference(mod, dy, x, ref, accumulate=accumulate, alpha=0.5)
        torch.cuda.synchronize()
        mod.read_errors()
        # Same kernel, same split and the same fixed summation order: bitwise equal.
        assert torch.equal(ours, ref), f"trial {trial}: max diff {(ours - ref).abs().max().item()}"
        exact = 0.5 * (dy.float().t() @ x.float()) + (init if accumulate else 0)
        err = (ours - exact).abs().max().item() / exact.abs().max().item()
        assert err < 1e-3, err


def _split(M, N, K, sms):
    """The split-K factor the GEMM launcher picks for an fp32 weight-gradient problem (its cost model:
    rounds of tiles times one slice's share of K, plus the fp32 partial products written and read)."""
    tiles = -(-M // 128) * -(-N // 256)
    if N < 256 or M % 4 or N % 4 or tiles >= 4 * sms:
        return 1
    num_kb = -(-K // 64)
    tile_s = 2.0 * 128 * 256 * K / 11e12
    slice_s = 8.0 * M * N / 6e12
    best, best_t = 1, -(-tiles // sms) * tile_s
    s = 2
    while s <= 16 and num_kb // s >= 16:
        t = -(-(tiles * s) // sms) * tile_s / s + s * slice_s
        if t < 0.98 * best_t:
            best, best_t = s, t
        s += 1
    return best


def _oversize_shape(sms, cap, K=16384):
    """(M, N) of a problem whose split-K partial products exceed the scratch on this GPU, or None."""
    for nt in range(1, 33):
        N = 256 * nt
        for mt in range(1, 2 * sms + 1):
            M = 128 * mt
            split = _split(M, N, K, sms)
            if split > 1 and split * M * N * 4 > cap:
                return M, N
    return None


def test_rejects_oversize_problem(lib):
    mod, fn, cap = lib
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    shape = _oversize_shape(sms, cap)
    if shape is None:
        pytest.skip(f"with {sms} SMs no split-K problem needs more than {cap} bytes of scratch")
    M, N = shape
    T = 16384
    dy = torch.zeros(T, M, device="cuda", dtype=torch.bfloat16)
    x = torch.zeros(T, N, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), 7.0, device="cuda")
    assert call(fn, dy, x, out, accumulate=False) == 1
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched


def test_allocates_nothing(lib):
    """A call, including the split-K scratch it uses, leaves the caching allocator untouched."""
    mod, fn, _ = lib
    T, N, K = 65536, 1280, 1280
    dy = torch.randn(T, N, device="cuda").to(torch.bfloat16)
    x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
    out = torch.zeros(N, K, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert _split(N, K, T, sms) > 1  # the scratch array is in use
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats()["allocation.all.allocated"]
    assert call(fn, dy, x, out, accumulate=False) == 0
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats()["allocation.all.allocated"] == before
    assert lib_error() == 0


def lib_error():
    from nexttransformer_b200.ops._ext import ext
    handle = ctypes.CDLL(ext().__file__)
    reader = handle.nt_wgrad_noalloc_read_error
    reader.restype = ctypes.c_int
    reader.argtypes = [ctypes.c_void_p]
    return reader(None)


def test_rejects_bad_arguments(lib):
    _, fn, _ = lib
    x = torch.zeros(64, 256, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(256, 256, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(None, 256, x.data_ptr(), 256, out.data_ptr(), 256, 256, 256, 64, 1.0, 0, stream) == 3
    assert fn(x.data_ptr() + 2, 256, x.data_ptr(), 256, out.data_ptr(), 256, 256, 256, 64, 1.0, 0, stream) == 3
    assert fn(x.data_ptr(), 255, x.data_ptr(), 256, out.data_ptr(), 256, 256, 256, 64, 1.0, 0, stream) == 3
