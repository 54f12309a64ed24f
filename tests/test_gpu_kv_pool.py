"""The KV page pool through the C ABI (tts_kv_pool_*), the allocator behind PagedKv: pages from
one pool per group of lanes, the reference's per-lane contiguous cache and broadcast-copied
shared prefix (crates/qwen3tts/src/qwen3.rs:122-212, 261-284) as block-table rows with shared
pages. Checks the device table rows and positions each admission writes, reference counts of
shared prefix pages, the copy of a partly filled page, refusals, and a decode state built from
the pool's own buffers."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def make_pool(tt, layers=2, n_kv=2, bs=4, blocks=12, lanes=3, max_blocks=4):
    from ttsnn import _lib as L
    desc = L.KvPoolDesc(layers, n_kv, 128, bs, blocks, lanes, max_blocks, None, None, None, None)
    h = C.c_void_p()
    L.call("tts_kv_pool_create", tt.ctx(0), C.byref(desc), C.byref(h))
    return L, L.load(), h


def lane_pages(lib, h, lane, cap=8):
    n = C.c_int(0)
    buf = (C.c_int * cap)()
    assert lib.tts_kv_pool_lane_pages(h, lane, buf, cap, C.byref(n)) == 0
    return list(buf[:n.value])


def device_state(L, lib, h, lanes):
    st = L.DecodeState()
    assert lib.tts_kv_pool_state(h, lanes, 0, C.byref(st)) == 0
    return st


def as_tensor(ptr, shape, dtype):
    """A torch view of device memory the pool owns (through __cuda_array_interface__)."""
    typestr = {torch.int32: "<i4", torch.float16: "<f2"}[dtype]

    class View:
        __cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                    "version": 3}
    return torch.as_tensor(View(), device="cuda")


def test_pool_admit_share_release(tt):
    L, lib, h = make_pool(tt)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.tts_kv_pool_free_pages(h) == 12
    assert lib.tts_kv_pool_admit(h, 0, 14, 9, stream) == 0  # 4 pages, 9 positions held
    p0 = lane_pages(lib, h, 0)
    assert p0 == [0, 1, 2, 3] and lib.tts_kv_pool_free_pages(h) == 8
    st = device_state(L, lib, h, 3)
    table = as_tensor(st.block_table, (3, 4), torch.int32)
    pos = as_tensor(st.positions, (3,), torch.int32)
    k = as_tensor(st.k_pages, (2, 12, 2, 4, 128), torch.float16)
    v = as_tensor(st.v_pages, (2, 12, 2, 4, 128), torch.float16)
    torch.cuda.synchronize()
    assert table[0].tolist() == p0 and pos[0].item() == 9
    # lane 0's pages hold distinct rows; lane 1 shares its first 9 positions: pages 0 and 1
    # shared, page 2 (1 of 4 rows used) copied, one more fresh page for capacity 13
    k.copy_(torch.randn_like(k, dtype=torch.float32).half())
    v.copy_(torch.randn_like(v, dtype=torch.float32).half())
    assert lib.tts_kv_pool_share_prefix(h, 0, 1, 9, 13, stream) == 0
    p1 = lane_pages(lib, h, 1)
    torch.cuda.synchronize()
    assert p1[:2] == [0, 1] and p1[2] not in p0 and len(p1) == 4
    assert table[1].tolist() == p1 and pos[1].item() == 9
    assert [lib.tts_kv_pool_page_refs(h, p) for p in p0] == [2, 2, 1, 1]
    assert torch.equal(k[:, p1[2]], k[:, p0[2]]) and torch.equal(v[:, p1[2]], v[:, p0[2]])
    # the shared pages stay until their last lane lets them go
    free = lib.tts_kv_pool_free_pages(h)
    assert lib.tts_kv_pool_release(h, 0) == 0
    assert lib.tts_kv_pool_free_pages(h) == free + 2  # pages 2 and 3 were lane 0's alone
    assert lib.tts_kv_pool_page_refs(h, 0) == 1
    assert lib.tts_kv_pool_release(h, 1) == 0
    assert lib.tts_kv_pool_free_pages(h) == 12 and lib.tts_kv_pool_page_refs(h, 0) == 0
    assert lib.tts_kv_pool_destroy(h) == 0


def test_pool_refusals(tt):
    L, lib, h = make_pool(tt, blocks=6)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.tts_kv_pool_admit(h, 0, 17, 0, stream) == 1  # 5 pages > max_blocks 4
    assert "table holds 4" in L.last_error()
    assert lib.tts_kv_pool_admit(h, 0, 16, 0, stream) == 0
    assert lib.tts_kv_pool_admit(h, 1, 12, 0, stream) == 5  # 3 pages, 2 free: OOM
    assert "exhausted" in L.last_error()
    assert lib.tts_kv_pool_admit(h, 3, 4, 0, stream) == 1  # lane outside 0..2
    busy = (C.c_int * 2)(0, 5)
    assert lib.tts_kv_pool_admit_pages(h, 2, busy, 2, 0, stream) == 1  # page 0 is lane 0's
    assert "not a free page" in L.last_error()
    mine = (C.c_int * 2)(5, 4)
    assert lib.tts_kv_pool_admit_pages(h, 2, mine, 2, 7, stream) == 0
    assert lane_pages(lib, h, 2) == [5, 4] and lib.tts_kv_pool_free_pages(h) == 0
    assert lib.tts_kv_pool_page_refs(h, 99) == -1
    assert lib.tts_kv_pool_destroy(h) == 0
