"""mrl_merge_topk (the device merge of per-shard exchange records) against merge_topk_host on the
same lists: identical ids and scores, including exact score ties across lists, short and empty lists,
and k smaller or larger than the live total."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _lists(rng, n_lists, stride, counts, levels):
    ids = np.zeros((n_lists, stride), np.uint64)
    sc = np.zeros((n_lists, stride), np.float32)
    for i in range(n_lists):
        c = counts[i]
        # distinct ids per shard (shard i owns block range [10000 i, 10000 i + 10000))
        blk = rng.choice(10000, size=c, replace=False) + 10000 * i
        v = ((blk << 16) | rng.integers(0, 64, size=c)).astype(np.uint64)
        s = rng.integers(0, levels, size=c).astype(np.float32) / levels  # many exact ties
        o = np.lexsort((v, -s.astype(np.float64)))
        ids[i, :c] = v[o]
        sc[i, :c] = s[o]
    return ids, sc


@pytest.mark.parametrize("n_lists,stride,k,levels", [(2, 256, 256, 7), (8, 256, 256, 1000), (8, 64, 300, 3),
                                                     (5, 4096, 4096, 50), (1, 16, 8, 4)])
def test_merge_matches_host(dev, n_lists, stride, k, levels):
    import torch

    import mrl_b200 as M

    rng = np.random.default_rng(n_lists * 7 + stride)
    counts = rng.integers(0, stride + 1, size=n_lists)
    counts[0] = stride
    if n_lists > 2:
        counts[1] = 0
    ids, sc = _lists(rng, n_lists, stride, counts, levels)
    d_rec = torch.from_numpy(M.pack_records(ids, sc, counts).reshape(-1)).cuda()
    o_ids = torch.full((k,), -1, dtype=torch.int64, device="cuda")
    o_sc = torch.zeros(k, dtype=torch.float32, device="cuda")
    o_cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    M._capi.check(dev.ptr, dev.lib.mrl_merge_topk(dev.ptr, C.c_void_p(d_rec.data_ptr()), n_lists, stride, k,
                                                  C.c_void_p(o_ids.data_ptr()), C.c_void_p(o_sc.data_ptr()),
                                                  C.c_void_p(o_cnt.data_ptr())))
    torch.cuda.synchronize()
    r_ids, r_sc = M.merge_topk_host(ids, sc, counts, k)
    n = int(o_cnt.item())
    assert n == len(r_ids)
    assert np.array_equal(o_ids.cpu().numpy()[:n].view(np.uint64), r_ids)
    assert np.array_equal(o_sc.cpu().numpy()[:n].view(np.uint32), r_sc.view(np.uint32))


def test_merge_rejects_bad_sizes(dev):
    import mrl_b200 as M

    z = C.c_void_p(16)
    for n_lists, stride, k in ((0, 16, 16), (2, 0, 16), (2, 16, 0), (2, 16, 5000), (2000, 16, 16)):
        rc = dev.lib.mrl_merge_topk(dev.ptr, z, n_lists, stride, k, z, z, z)
        assert rc == M._capi.MRL_ERR_INVALID
    assert dev.lib.mrl_merge_topk(dev.ptr, C.c_void_p(24), 2, 16, 16, z, z, z) == M._capi.MRL_ERR_INVALID
