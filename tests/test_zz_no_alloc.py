"""The allocation-free commitment entry point (uwc_b3_root_and_seed_noalloc).

It exists for callers that cannot allocate device memory when they commit to a matrix: code
running under CUDA graph capture, foreign-function callers with no device allocator, processes
whose device memory another framework has reserved. It keeps its scratch in a fixed array of
the library's device memory, so this file checks, through the C ABI, that two calls in a row
give exactly the root and seed of the regular entry point (which takes caller scratch), and
that inputs beyond the fixed array's limit are refused. The file is named to run last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _commit(L, data, key, prefix, salt, dim, noalloc):
    root = torch.zeros(8, dtype=torch.int32, device="cuda")
    seed = torch.zeros(8, dtype=torch.int32, device="cuda")
    nbytes = data.numel()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = L.uwc_b3_root_and_seed_noalloc(_ptr(data), nbytes, _ptr(key), _ptr(prefix), _ptr(salt), dim, _ptr(root),
                                            _ptr(seed), stream)
    else:
        words = L.uwc_b3_scratch_words(nbytes)
        scratch = torch.empty(words, dtype=torch.int32, device="cuda")
        rc = L.uwc_b3_root_and_seed(_ptr(data), nbytes, _ptr(key), _ptr(prefix), _ptr(salt), dim, _ptr(root),
                                    _ptr(seed), _ptr(scratch), words, stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return root.cpu().numpy(), seed.cpu().numpy()


def test_noalloc_commitment_matches_regular_entry_point(dev):
    from uwc_b200 import _lib
    L = _lib.lib()
    _lib.device_status(clear=True)
    gen = torch.Generator(device="cuda").manual_seed(77)
    key = torch.randint(-2 ** 31, 2 ** 31 - 1, (8,), dtype=torch.int32, device="cuda", generator=gen)
    prefix = torch.randint(-2 ** 31, 2 ** 31 - 1, (8,), dtype=torch.int32, device="cuda", generator=gen)
    salt = torch.randint(-2 ** 31, 2 ** 31 - 1, (8,), dtype=torch.int32, device="cuda", generator=gen)
    max_bytes = int(L.uwc_b3_noalloc_max_bytes())
    assert max_bytes == 128 << 20
    key_bytes = key.cpu().numpy().astype("<i4").tobytes()
    # calls in a row on different inputs: the shared scratch keeps the previous call's contents
    # when the next runs, and the next must not depend on them. The sizes cover the largest input
    # (1024 chunk groups, one reduce level), a ragged group count, a single full group (the chunk
    # kernel applies ROOT at its own merge) and a single chunk (ROOT on the chunk compression).
    for nbytes, dim in ((max_bytes, 8192), (3 * 1024 * 129, 387), (128 * 1024, 64), (1024, 1)):
        data = torch.randint(-128, 128, (nbytes,), dtype=torch.int8, device="cuda", generator=gen)
        want_root, want_seed = _commit(L, data, key, prefix, salt, dim, noalloc=False)
        got_root, got_seed = _commit(L, data, key, prefix, salt, dim, noalloc=True)
        assert np.array_equal(got_root, want_root) and np.array_equal(got_seed, want_seed), nbytes
        if nbytes <= 1 << 20:
            import blake3
            digest = blake3.blake3(data.cpu().numpy().tobytes(), key=key_bytes).digest()
            assert got_root.astype("<i4").tobytes() == digest, nbytes
    assert _lib.device_status(clear=True) == 0


def test_noalloc_refuses_inputs_beyond_its_scratch(dev):
    from uwc_b200 import _lib
    L = _lib.lib()
    fake = ctypes.c_void_p(0x1000)   # refused before any device access
    rc = L.uwc_b3_root_and_seed_noalloc(fake, int(L.uwc_b3_noalloc_max_bytes()) + 1024, fake, fake, fake, 1, None,
                                        fake, None)
    assert rc == _lib.ERR_SCRATCH
    assert L.uwc_b3_root_and_seed_noalloc(fake, 1000, fake, None, None, 0, fake, None, None) == _lib.ERR_SHAPE
