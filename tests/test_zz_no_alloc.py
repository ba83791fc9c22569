"""The allocation-free attention entry point against the regular one.

qasr_kernel_attention_noalloc serves callers that cannot call cudaMalloc (hosts with a
fixed memory budget, real-time audio callbacks that must not block on the allocator):
its scratch and status word are static device arrays.  This file is collected last on
purpose, so a run that stops at the first failure has already run every other test; it
must also pass alone in a fresh process, where its first call performs the one-time
symbol lookup.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the attention parity tolerance of tests/test_gpu_kernels.py


def _inputs(torch, seed, lens, nkv=8, layers=1, layer=0):
    rng = np.random.default_rng(seed)
    rows = len(lens)
    max_pages = max((l + 63) // 64 for l in lens)
    n_pages = rows * max_pages
    pt = rng.permutation(n_pages).astype(np.int32).reshape(rows, max_pages)
    pool = (rng.standard_normal((n_pages, layers, 2, nkv, 64, 128)).astype(np.float16))
    q = rng.standard_normal((rows, 2 * nkv * 128)).astype(np.float16)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dict(q=dev(q), pool=dev(pool), pt=dev(pt), rs=dev(np.arange(rows, dtype=np.int32)),
                rp=dev(np.array([l - 1 for l in lens], np.int32)), rows=rows, max_pages=max_pages,
                nkv=nkv, layers=layers, layer=layer)


def _run(fn, torch, t):
    out = torch.zeros_like(t["q"])
    fn(0, 0, t["q"].data_ptr(), 2 * t["nkv"] * 128, out.data_ptr(), t["pool"].data_ptr(), t["pt"].data_ptr(),
       t["max_pages"], t["layers"], t["nkv"], t["layer"], t["rs"].data_ptr(), t["rp"].data_ptr(), t["rows"])
    torch.cuda.synchronize()
    return out.cpu().numpy().astype(np.float32)


def test_noalloc_attention_matches_regular_entry_point(qasr, cuda_device):
    import torch
    # lengths that split rows into several chunks (merge through the scratch) and not
    lens = [1, 63, 64, 65, 300, 700, 1500, 2048, 4000] + [17 * i + 5 for i in range(20)]
    t = _inputs(torch, 11, lens)
    want = _run(qasr.kernel_attention, torch, t)
    for call in range(2):  # two calls in a row: the scratch keeps the last call's contents
        got = _run(qasr.kernel_attention_noalloc, torch, t)
        err = np.max(np.abs(got - want) / (np.abs(want) + 0.05))
        assert err <= TOL, f"call {call}: relative error {err}"


def test_noalloc_attention_rejects_oversize(qasr, cuda_device):
    import torch
    t = _inputs(torch, 3, [10] * 65, layers=1, layer=0)
    with pytest.raises(qasr.DecoderError) as e:
        _run(qasr.kernel_attention_noalloc, torch, t)
    assert e.value.status == 3 and "64 query rows" in str(e.value)
