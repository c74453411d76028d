"""GPU test of the allocation-free C entry point `bdh_decoder_merge_noalloc`.

That entry point exists for callers that may not allocate device memory themselves — a
runtime that plans all memory up front and forbids allocation while it runs, a plugin
living inside a framework that owns the CUDA allocator, or plain C code calling this
library through an FFI with no PyTorch allocator. Its scratch is a fixed array compiled
into the library. The test calls it through its exported C symbol (ctypes) twice in a
row, with different inputs, and compares each result with the regular path (split-K
GEMM into a torch-allocated partial buffer, then the rowwise.cu residual-merge kernel).

The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from burn_dragon_b200 import _ext

    lib = ctypes.CDLL(_ext.load()._mod.__file__)
    fn = lib.bdh_decoder_merge_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.bdh_noalloc_error_string.restype = ctypes.c_char_p
    lib.bdh_noalloc_error_string.argtypes = [ctypes.c_int]
    lib.bdh_noalloc_error_word.restype = ctypes.c_void_p
    lib.bdh_noalloc_error_word.argtypes = []
    return lib, fn


def _real_splits(N, splits):
    """The split count the entry point uses: K-blocks per split rounded up, then the
    number of splits that covers N / 64 K-blocks."""
    kb = N // 64
    per = -(-kb // splits)
    return -(-kb // per)


def _regular_path(yn, dec, v, gamma, beta, splits, eps):
    from burn_dragon_b200 import _ext
    from burn_dragon_b200.ops import gemm as G

    M, N = yn.shape
    D = dec.shape[1]
    partial = torch.empty(splits, M, D, device=yn.device)
    G.gemm(G.EPI_F32, G.Operand(yn, False, N, M, N), G.Operand(dec, True, D, N, D), M, D, N, partial,
           splits=splits, ld=D, split_stride=M * D)
    out = torch.empty(M, D, device=yn.device)
    _ext.load().tail_fwd(partial, splits, M * D, v, M, D, gamma, beta, eps, None, out, None, None)
    return out


@pytest.mark.parametrize("M,N,D,splits", [(256, 2048, 256, 4), (384, 1024, 128, 2),
                                          # D narrower than a 128-wide tile, row tails (M % 128 != 0) and a
                                          # split count that rounds down (5 -> 4 over 16 K-blocks)
                                          (200, 512, 64, 3), (130, 1024, 32, 5)])
def test_noalloc_matches_regular_entry_point_twice(M, N, D, splits):
    lib, fn = _lib()
    eps = 1e-5
    stream = torch.cuda.current_stream()
    for call in range(2):
        torch.manual_seed(100 + call)
        yn = torch.relu(torch.randn(M, N, device="cuda")).bfloat16()
        dec = (torch.randn(N, D, device="cuda") * 0.05).bfloat16()
        v = torch.randn(M, D, device="cuda")
        gamma = 1.0 + 0.1 * torch.randn(D, device="cuda")
        beta = 0.1 * torch.randn(D, device="cuda")
        out = torch.full((M, D), float("nan"), device="cuda")
        out16 = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
        rc = fn(yn.data_ptr(), dec.data_ptr(), v.data_ptr(), gamma.data_ptr(), beta.data_ptr(), out.data_ptr(),
                out16.data_ptr(), M, N, D, splits, eps, 1, stream.cuda_stream)
        assert rc == 0, lib.bdh_noalloc_error_string(rc).decode()
        ref = _regular_path(yn, dec, v, gamma, beta, _real_splits(N, splits), eps)
        torch.cuda.synchronize()
        err = (out - ref).abs().max().item()
        assert err < 2e-3, f"call {call}: max abs err {err}"
        assert (out16.float() - ref).abs().max().item() < 3e-2


def test_noalloc_rejects_oversized_request():
    lib, fn = _lib()
    M, N, D = 16384, 32768, 256  # 4 splits * 16384 * 256 * 4 B = 64 MiB > 32 MiB scratch
    x = torch.empty(8, device="cuda")
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), None, M, N, D, 4,
            1e-5, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 2, lib.bdh_noalloc_error_string(rc).decode()


def test_noalloc_error_word_is_clear_after_an_unchecked_call():
    lib, fn = _lib()
    M, N, D = 128, 512, 128
    torch.manual_seed(7)
    yn = torch.relu(torch.randn(M, N, device="cuda")).bfloat16()
    dec = (torch.randn(N, D, device="cuda") * 0.05).bfloat16()
    v = torch.randn(M, D, device="cuda")
    gamma, beta = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
    out = torch.empty(M, D, device="cuda")
    rc = fn(yn.data_ptr(), dec.data_ptr(), v.data_ptr(), gamma.data_ptr(), beta.data_ptr(), out.data_ptr(), None,
            M, N, D, 2, 1e-5, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.bdh_noalloc_error_string(rc).decode()
    addr = lib.bdh_noalloc_error_word()
    assert addr
    from burn_dragon_b200 import _ext

    word = _ext.load().wrap_ptr(addr, 1, 2, torch.cuda.current_device())  # a view of the device int
    torch.cuda.synchronize()
    assert int(word.item()) == 0
