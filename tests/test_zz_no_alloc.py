"""The allocation-free decode-attention entry point, called through its exported C symbol.

For callers that must not allocate device memory (hosts whose memory manager owns the whole
device budget, allocator-free serving loops): the split-KV scratch lives in a fixed static device
array inside the library. These tests call ``gollek_paged_decode_attention_noalloc`` (declared in
csrc/kernels/noalloc.h) with ctypes on raw device pointers and check it against the regular entry
point (``ops.paged_decode_attention``, which takes its scratch from the caller) and against the
fp32 paged-attention oracle, on two consecutive calls; then the other head sizes, the unsplit
path, and the error codes for an oversized request, an unsupported shape and bad arguments.

Collected last on purpose (``zz``), so that a failure here cannot stop the rest of the suite.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from gollek_b200.native import _so_path, cuda_ext
    cuda_ext()  # loads the module (and libtorch) first
    lib = ctypes.CDLL(_so_path("gollek_b200_C"))
    f = lib.gollek_paged_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
    cap = lib.gollek_paged_decode_attention_noalloc_scratch_bytes
    cap.restype = ctypes.c_size_t
    return f, int(cap())


def _case(seed, B, Hk, G, D, lens):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bs = 16
    max_blocks = max((l + bs - 1) // bs for l in lens)
    NB = B * max_blocks + 2
    cache = torch.randn(NB, 2, Hk, bs, D, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(NB, device="cuda", generator=g).int()
    bt = torch.zeros(B, max_blocks, dtype=torch.int32, device="cuda")
    k = 0
    for b, l in enumerate(lens):
        n = (l + bs - 1) // bs
        bt[b, :n] = perm[k:k + n]
        k += n
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hk * G, D, device="cuda", generator=g).bfloat16()
    return q, cache, bt, sl


def _call(f, q, cache, bt, sl, splits, scale, out):
    B, H, D = q.shape
    Hk, bs = cache.shape[2], cache.shape[3]
    return f(out.data_ptr(), q.data_ptr(), q.stride(0), cache.data_ptr(), cache.shape[0], bt.data_ptr(), bt.stride(0),
             sl.data_ptr(), B, H, Hk, D, bs, splits, scale, torch.cuda.current_stream().cuda_stream)


def _oracle(q, cache, bt, sl, scale):
    """fp32 paged attention of one query per sequence (ops/reference.py)."""
    from gollek_b200.ops import reference as ref_ops
    B = q.shape[0]
    qsl = torch.arange(B + 1, dtype=torch.int32, device=q.device)
    return ref_ops.paged_attention(q.float(), cache.float(), bt, sl, qsl, scale)


def test_noalloc_decode_matches_regular_entry_point_twice():
    from gollek_b200 import ops
    f, cap = _lib()
    assert cap == 8 << 20
    for call, (seed, lens, splits) in enumerate([(1, [5, 300, 1029, 64], 4), (2, [700, 17, 2048], 8)]):
        q, cache, bt, sl = _case(seed, len(lens), 2, 4, 128, lens)
        scale = 1 / math.sqrt(128)
        out = torch.empty_like(q)
        rc = _call(f, q, cache, bt, sl, splits, scale, out)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: error code {rc}"
        ref = ops.paged_decode_attention(q, cache, bt, sl, scale, num_splits=splits)
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(out.float(), _oracle(q, cache, bt, sl, scale), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("D,G,splits", [(64, 4, 4), (256, 2, 3), (128, 8, 1), (64, 1, 1)])
def test_noalloc_other_head_sizes_and_unsplit(D, G, splits):
    f, _ = _lib()
    lens = [33, 517, 16]
    q, cache, bt, sl = _case(10 + D + G, len(lens), 2, G, D, lens)
    scale = 1 / math.sqrt(D)
    for _ in range(2):  # the second call reuses the scratch left by the first
        out = torch.empty_like(q)
        rc = _call(f, q, cache, bt, sl, splits, scale, out)
        torch.cuda.synchronize()
        assert rc == 0, rc
        torch.testing.assert_close(out.float(), _oracle(q, cache, bt, sl, scale), rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_unsupported_and_bad_arguments():
    f, _ = _lib()
    q, cache, bt, sl = _case(4, 2, 2, 4, 128, [40, 50])
    out = torch.empty_like(q)
    B, H, D = q.shape

    def call(**kw):
        a = dict(H=H, Hk=2, D=D, bs=16, splits=2)
        a.update(kw)
        return f(out.data_ptr(), q.data_ptr(), q.stride(0), cache.data_ptr(), cache.shape[0], bt.data_ptr(),
                 bt.stride(0), sl.data_ptr(), B, a["H"], a["Hk"], a["D"], a["bs"], a["splits"], 0.088,
                 torch.cuda.current_stream().cuda_stream)

    assert call(bs=32) == 4          # block size the kernels are not built for
    assert call(D=96) == 4           # head size without a kernel
    assert call(H=8, Hk=3) == 1      # H not a multiple of Hk
    assert call(splits=0) == 1
    assert f(0, q.data_ptr(), q.stride(0), cache.data_ptr(), cache.shape[0], bt.data_ptr(), bt.stride(0),
             sl.data_ptr(), B, H, 2, D, 16, 2, 0.088, 0) == 1  # null output
    torch.cuda.synchronize()  # nothing was launched; the context is untouched


def test_noalloc_rejects_oversized_request():
    f, cap = _lib()
    B, H, D, splits = 64, 64, 128, 32  # 64*64*32*130*4 bytes > 8 MiB
    assert B * H * splits * (D + 2) * 4 > cap
    q, cache, bt, sl = _case(3, 2, 8, 8, D, [40, 50])
    out = torch.empty_like(q)
    rc = f(out.data_ptr(), q.data_ptr(), q.stride(0), cache.data_ptr(), cache.shape[0], bt.data_ptr(),
           bt.stride(0), sl.data_ptr(), B, H, 8, D, 16, splits, 0.088, 0)
    assert rc == 2
