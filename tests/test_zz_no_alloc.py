"""The allocation-free decode-attention entry point, called through its
exported C symbol, gives the same output as the regular entry point (which
takes its workspace from PyTorch's allocator) on two calls in a row.

Collected last on purpose (test_zz_*): if it fails, a run that stops at the
first failure has already run every other test. Passes alone in a fresh
process and after the rest of the suite."""
import ctypes
import math

import pytest
import torch

from deltaserve_vllm_b200 import ops

pytestmark = pytest.mark.gpu


def _lib():
    assert ops.native_available(), ops._C_ERR
    lib = ctypes.CDLL(ops._EXT.__file__)
    fn = lib.dsv_paged_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p]
    return fn


def _case(seed, lens, Hq, Hkv, bs=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nb = sum(-(-l // bs) for l in lens) + 2
    kc = torch.randn(nb, Hkv, bs, 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(nb, Hkv, bs, 128, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(nb, device="cpu").tolist()
    maxb = max(-(-l // bs) for l in lens)
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    k = 0
    for i, l in enumerate(lens):
        n = -(-l // bs)
        bt[i, :n] = torch.tensor(perm[k:k + n])
        k += n
    q = torch.randn(len(lens), Hq * 128, generator=g, device="cuda").to(torch.bfloat16)
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("Hq,Hkv,lens,even", [(32, 8, [1, 600, 2049, 77], False), (16, 8, [300, 5, 1024], False),
                                               (32, 8, [1, 600, 2049, 77], True)])
def test_noalloc_decode_matches_regular_entry_point(Hq, Hkv, lens, even):
    """``even``: keys_per_split 0, each sequence splits its own context."""
    fn = _lib()
    scale = 1 / math.sqrt(128)
    for call, seed in enumerate((1, 2)):  # two calls in a row share the scratch array
        q, kc, vc, bt, ctx = _case(seed + 10 * Hq, lens, Hq, Hkv)
        splits, kps = ops.decode_splits(len(lens), Hkv, max(lens))
        if even:
            kps = 0
        exp = torch.zeros(len(lens), Hq * 128, dtype=torch.bfloat16, device="cuda")
        po = torch.empty(len(lens) * Hq * splits * 128, device="cuda")
        pml = torch.empty(len(lens) * Hq * splits * 2, device="cuda")
        ops.paged_decode(q, kc, vc, bt, ctx, exp, Hq, scale, po, pml, splits, kps)
        got = torch.zeros_like(exp)
        stream = torch.cuda.current_stream()
        rc = fn(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), Hkv, kc.shape[2], bt.data_ptr(),
                bt.shape[1], ctx.data_ptr(), len(lens), got.data_ptr(), got.stride(0), Hq, scale, splits, kps,
                stream.cuda_stream)
        assert rc == 0, f"call {call}: rc={rc}"
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), exp.float(), rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_oversized_request():
    fn = _lib()
    q, kc, vc, bt, ctx = _case(5, [64], 32, 8)
    got = torch.zeros(1, 32 * 128, dtype=torch.bfloat16, device="cuda")
    # 1 x 32 heads x 512 splits x 130 floats > 4 MiB of scratch
    rc = fn(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), 8, 64, bt.data_ptr(), bt.shape[1],
            ctx.data_ptr(), 1, got.data_ptr(), got.stride(0), 32, 0.1, 512, 64,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
