"""GPU test of ``kiv_retrieve_attend_noalloc``, the entry point that allocates nothing.

Some callers cannot allocate device memory at the time they run a decode step:
a serving engine that gives all GPU memory to its own KV-block pool at start-up
and forbids cudaMalloc afterwards, or a plugin host whose custom-op interface
offers no allocator or workspace.  For them the library keeps a fixed scratch
array on every GPU and this entry point uses it instead of a caller workspace.

The test builds a cold store through the public Python surface, then calls the
existing entry point (``kiv_retrieve_attend`` with a freshly zeroed caller
workspace) and the allocation-free one through the C ABI, twice with
different queries -- with a call of another query shape in between, whose
data the shared scratch keeps -- and checks that outputs agree within the
fp32 tolerance used by the other parity tests and that the selected token
sets are identical.  This file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch
from transformers import PretrainedConfig

from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
from kiv_b200 import _native as nat

pytestmark = pytest.mark.gpu

RTOL = 1e-5   # fp32 output tolerance of the parity tests


def _store():
    dev = torch.device("cuda:0")
    cfg = KIVConfig(hot_budget=256, page_size=128, top_pages=8, top_p=128, telemetry=False)
    topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=8, num_kv_heads=2,
                                head_dim=64, num_hidden_layers=1)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, dev)
    g = torch.Generator(device=dev).manual_seed(11)
    k = torch.randn(1, 2, 6000, 64, generator=g, device=dev)
    v = torch.randn(1, 2, 6000, 64, generator=g, device=dev)
    cache.update(k, v, 0)
    cache.mark_prefill_complete()
    return cfg, cache.get_cold_store(0), g


def _call_both(lib, desc, store, cfg, q, md, stream, top_pages=None):
    """kiv_retrieve_attend with a freshly zeroed workspace, then the allocation-free
    entry point, on the same query; returns both selections and outputs."""
    dev = store.device
    tp = cfg.top_pages if top_pages is None else top_pages
    qd = nat.query_desc(q, 0.125, tp, cfg.top_p)
    nbytes = lib.kiv_workspace_bytes(ctypes.byref(desc), ctypes.byref(qd))
    ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
    ws = ws[(-ws.data_ptr()) % 256:][:nbytes]
    Q = q.shape[2]
    sel_a = torch.zeros(1, cfg.top_p, dtype=torch.int32, device=dev)
    sel_b = torch.zeros_like(sel_a)
    out_a = torch.zeros(1, Q, 8, 64, device=dev)
    out_b = torch.zeros_like(out_a)
    rc = lib.kiv_retrieve_attend(ctypes.byref(desc), ctypes.byref(qd), ctypes.byref(md),
                                 ws.data_ptr(), nbytes, 0, sel_a.data_ptr(), out_a.data_ptr(), stream)
    nat.check(rc, "retrieve_attend")
    torch.cuda.synchronize(dev)
    before = torch.cuda.memory_allocated(dev)
    rc = lib.kiv_retrieve_attend_noalloc(ctypes.byref(desc), ctypes.byref(qd), ctypes.byref(md),
                                         sel_b.data_ptr(), out_b.data_ptr(), stream)
    nat.check(rc, "retrieve_attend_noalloc")
    torch.cuda.synchronize(dev)
    assert torch.cuda.memory_allocated(dev) == before
    return sel_a, sel_b, out_a, out_b


def test_noalloc_matches_workspace_entry_point_twice():
    cfg, store, g = _store()
    lib = nat.load_library()
    dev = store.device
    desc = store.descriptor()
    desc.hot_hint = store.hot_length
    md = nat.mask_desc(None, False)
    stream = torch.cuda.current_stream(dev).cuda_stream
    P = min(cfg.top_p, store.cold_length)
    for call in range(2):
        if call == 1:
            # a call of another shape (2 query positions, fewer pages per row)
            # between the two checked calls leaves its own data in the scratch
            q2 = torch.randn(1, 8, 2, 64, generator=g, device=dev)
            _call_both(lib, desc, store, cfg, q2, md, stream, top_pages=4)
        q = torch.randn(1, 8, 1, 64, generator=g, device=dev)
        sel_a, sel_b, out_a, out_b = _call_both(lib, desc, store, cfg, q, md, stream)
        assert set(sel_a[0, :P].tolist()) == set(sel_b[0, :P].tolist()), f"call {call}"
        a, b = out_a.double().cpu().numpy(), out_b.double().cpu().numpy()
        assert np.abs(a - b).max() <= RTOL * np.abs(a).max(), f"call {call}"


def test_noalloc_rejects_shapes_beyond_the_scratch():
    cfg, store, g = _store()
    lib = nat.load_library()
    desc = store.descriptor()
    huge = nat.StoreDesc.from_buffer_copy(desc)
    huge.cold_capacity = 1 << 28          # 2M pages: coarse scores alone need 64 MiB
    q = torch.randn(1, 8, 1, 64, device=store.device)
    qd = nat.query_desc(q, 0.125, 64, 1024)
    sel = torch.zeros(1, 1024, dtype=torch.int32, device=store.device)
    out = torch.zeros(1, 1, 8, 64, device=store.device)
    rc = lib.kiv_retrieve_attend_noalloc(ctypes.byref(huge), ctypes.byref(qd), None, sel.data_ptr(),
                                         out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert b"scratch" in lib.kiv_last_error()
