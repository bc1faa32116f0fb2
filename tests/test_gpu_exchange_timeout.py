"""The bounded wait of the peer-memory exchange gives up, reports, and writes nothing.

One GPU plays rank 0 of a world of 2: the second "rank's" arena is a plain
local buffer that no process ever writes, so every wait on rank 1's data runs
out -- the attention merge waiting for rank 1's partials, and the candidate
exchange's select waiting for the keys of the pages rank 1 owns.  With a wait
bound of about a millisecond (``kiv_exchange.wait_cycles``) the call must
return promptly, set KIV_ERRBIT_WAIT_TIMEOUT in the store's state and write no
result (the merge leaves its output untouched, the select selects nothing);
the context stays usable (a second call behaves the same way, and an ordinary
kernel runs afterwards).  Nothing faults, traps or hangs: the flag that is
never set is the only failure.
"""

import ctypes
import time

import pytest
import torch

from kiv_b200 import _native as nat

pytestmark = pytest.mark.gpu

WAIT_CYCLES = 2_000_000      # about 1 ms at the B200's 1965 MHz SM clock


def _descs(dev):
    B, HKV, D, HQ = 1, 1, 64, 8
    state = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device=dev)
    st = nat.StoreDesc(B, HKV, D, 128, nat.KIV_DTYPE[torch.float32], 0, 2, 0, 0, 0,
                       None, None, None, None, None, state.data_ptr(), 0, None, None, 0, 0)
    q = torch.zeros(B, HQ, 1, D, device=dev)
    qd = nat.query_desc(q, 0.125, 4, 64)
    return st, qd, q, state


def test_exchange_wait_runs_out_and_reports():
    dev = torch.device("cuda:0")
    L = nat.load_library()
    st, qd, q, state = _descs(dev)
    nbytes = L.kiv_exchange_bytes(ctypes.byref(st), ctypes.byref(qd), 2)
    assert nbytes > 0
    own = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
    silent = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)   # "rank 1": nobody writes it
    a0 = own.data_ptr() + (-own.data_ptr()) % 256
    a1 = silent.data_ptr() + (-silent.data_ptr()) % 256
    arenas = (ctypes.c_void_p * nat.MAX_PEERS)(a0, a1)
    x = nat.ExchangeDesc(2, 0, arenas, nbytes, WAIT_CYCLES)
    R = 8
    partial = torch.randn(R, 64 + 4, device=dev)
    out = torch.full((1, 1, 8, 64), 7.0, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        state.zero_()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        nat.check(L.kiv_attend_exchange_merge(ctypes.byref(st), ctypes.byref(qd), partial.data_ptr(),
                                              ctypes.byref(x), out.data_ptr(), s), "attend_exchange_merge")
        torch.cuda.synchronize(dev)
        el = time.perf_counter() - t0
        assert el < 0.5, f"call {call}: the bounded wait took {el:.3f} s"
        assert int(state[nat.ST_ERROR]) & 8, f"call {call}: KIV_ERRBIT_WAIT_TIMEOUT not set"
        assert torch.all(out == 7.0), f"call {call}: output written after a failed exchange"
    # the context is still usable
    y = torch.arange(1024, device=dev, dtype=torch.float32).sum()
    assert float(y) == 1023 * 1024 / 2


def test_exchange_rejects_negative_wait_bound():
    dev = torch.device("cuda:0")
    L = nat.load_library()
    st, qd, q, state = _descs(dev)
    nbytes = L.kiv_exchange_bytes(ctypes.byref(st), ctypes.byref(qd), 2)
    own = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
    a0 = own.data_ptr() + (-own.data_ptr()) % 256
    x = nat.ExchangeDesc(2, 0, (ctypes.c_void_p * nat.MAX_PEERS)(a0, a0), nbytes, -1)
    partial = torch.zeros(8, 68, device=dev)
    out = torch.zeros(1, 1, 8, 64, device=dev)
    rc = L.kiv_attend_exchange_merge(ctypes.byref(st), ctypes.byref(qd), partial.data_ptr(), ctypes.byref(x),
                                     out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 1


class _SilentPeer:
    """Exchange provider of a 2-rank page-sharded store on one GPU: rank 1's
    arena is a local buffer that nothing ever writes."""

    size, rank = 2, 0

    def __init__(self):
        self.bufs = []

    def exchange(self, nbytes, device):
        own = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        silent = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        self.bufs += [own, silent]
        arenas = [t.data_ptr() + (-t.data_ptr()) % 256 for t in (own, silent)]
        return nat.ExchangeDesc(2, 0, (ctypes.c_void_p * nat.MAX_PEERS)(*arenas), nbytes, WAIT_CYCLES)


def test_candidate_exchange_wait_runs_out_and_selects_nothing():
    from kiv_b200 import ColdKVStore, KIVConfig, ModelTopology

    dev = torch.device("cuda:0")
    cfg = KIVConfig(hot_budget=256, page_size=128, top_pages=4, top_p=64, telemetry=False)
    topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=8, num_kv_heads=1, head_dim=128,
                                num_hidden_layers=1)
    store = ColdKVStore(cfg, topo, dev, shard_rank=0, shard_count=2, comm=_SilentPeer())
    assert store.replicated_summaries
    g = torch.Generator(device=dev).manual_seed(5)
    k = torch.randn(1, 1, 6 * 128 + 9, 128, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 1, 6 * 128 + 9, 128, device=dev, generator=g).to(torch.bfloat16)
    store.evict_from_hot(k, v)        # 6 pages + 9 tokens; every shard sees every row
    q = torch.randn(1, 8, 1, 128, device=dev, generator=g).to(torch.bfloat16)
    qd = nat.query_desc(q, 0.1, cfg.top_pages, cfg.top_p)
    assert nat.lib().kiv_fine_exchange_supported(ctypes.byref(store.descriptor()), ctypes.byref(qd)) == 1
    for call in range(2):
        store._state[nat.ST_ERROR] = 0
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        store.retrieve_indices(q, 0.1, cfg)
        torch.cuda.synchronize(dev)
        el = time.perf_counter() - t0
        assert el < 0.5, f"call {call}: the bounded wait took {el:.3f} s"
        st = store.read_state()
        assert st[nat.ST_ERROR] & 8, f"call {call}: KIV_ERRBIT_WAIT_TIMEOUT not set"
        assert st[nat.ST_SEL] == 0 and st[nat.ST_SEL_LOCAL] == 0, f"call {call}: rows selected after a failed exchange"
    y = torch.arange(1024, device=dev, dtype=torch.float32).sum()
    assert float(y) == 1023 * 1024 / 2
