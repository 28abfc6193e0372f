"""mg_sort_pairs_u32_noalloc: the radix sort for callers that cannot allocate
device memory (a host that hands the library no allocator, or owns the whole
GPU through its own pool), with its scratch in a static array inside the
library. Called through the C ABI and checked against mg_sort_pairs_u32 (the
entry point that takes caller scratch) on two calls in a row, the second with
an odd number of digit passes so the result comes back from the static
ping-pong buffers. Integer data: the results must be identical.

This file is collected last on purpose: run alone in a fresh process or after
the whole suite, it must pass either way."""

import ctypes as C

import numpy as np
import pytest
import torch

from metal_gauss_b200 import _lib, ext

pytestmark = pytest.mark.gpu

MAX_N = 1 << 20


def _noalloc(keys: torch.Tensor, vals: torch.Tensor, bits: int) -> None:
    lib = _lib.load()
    status = lib.mg_sort_pairs_u32_noalloc(keys.data_ptr(), vals.data_ptr(), keys.numel(), bits,
                                           torch.cuda.current_stream().cuda_stream)
    assert status == 0, lib.mg_last_error().decode()


def _case(n: int, bits: int, seed: int, ties: int):
    g = np.random.default_rng(seed)
    keys = g.integers(0, ties, n).astype(np.uint32) & np.uint32((1 << bits) - 1 if bits < 32
                                                                else 0xFFFFFFFF)
    vals = g.integers(0, 1 << 31, n).astype(np.uint32)
    return keys, vals


def test_noalloc_sort_matches_the_scratch_entry_point_twice(cuda):
    cases = [(1_000_000, 32, 1, 1 << 31), (300_001, 20, 2, 1 << 14)]   # 4 passes, then 3
    for n, bits, seed, ties in cases:
        keys, vals = _case(n, bits, seed, ties)
        k = torch.from_numpy(keys.view(np.int32)).cuda()
        v = torch.from_numpy(vals.view(np.int32)).cuda()
        _noalloc(k, v, bits)
        ref_k, ref_v = ext.sort_pairs(torch.from_numpy(keys.view(np.int32)).cuda(),
                                      torch.from_numpy(vals.view(np.int32)).cuda(), bits)
        torch.cuda.synchronize()
        assert torch.equal(k, ref_k) and torch.equal(v, ref_v)
        order = np.argsort(keys, kind="stable")
        assert np.array_equal(k.cpu().numpy().view(np.uint32), keys[order])
        assert np.array_equal(v.cpu().numpy().view(np.uint32), vals[order])
    assert ext.device_error() == 0


@pytest.mark.parametrize("n,bits", [(MAX_N, 32), (200_003, 8)])
def test_noalloc_sort_at_its_maximum_and_with_one_pass(cuda, n, bits):
    """Exactly MAX_N pairs (the static look-back region used to its last
    word), and an 8-bit key (one pass: the result comes back from the static
    buffers)."""
    keys, vals = _case(n, bits, 5 + bits, 1 << 31)
    k = torch.from_numpy(keys.view(np.int32)).cuda()
    v = torch.from_numpy(vals.view(np.int32)).cuda()
    _noalloc(k, v, bits)
    ref_k, ref_v = ext.sort_pairs(torch.from_numpy(keys.view(np.int32)).cuda(),
                                  torch.from_numpy(vals.view(np.int32)).cuda(), bits)
    torch.cuda.synchronize()
    assert torch.equal(k, ref_k) and torch.equal(v, ref_v)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(v.cpu().numpy().view(np.uint32), vals[order])
    assert ext.device_error() == 0


def test_noalloc_sort_rejects_sizes_beyond_its_maximum(cuda):
    lib = _lib.load()
    k = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = lib.mg_sort_pairs_u32_noalloc(k.data_ptr(), k.data_ptr(), MAX_N + 1, 32,
                                           torch.cuda.current_stream().cuda_stream)
    assert status == 2                                          # MG_ERR_CAPACITY
    assert b"MG_SORT_NOALLOC_MAX_N" in lib.mg_last_error()
