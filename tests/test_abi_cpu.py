"""CPU checks of the C ABI: the library loads, exports every declared entry
point, its structs have the header's layout, and argument validation rejects
bad calls before anything is launched (no GPU needed)."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from kiv_b200 import _native as nat

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kiv_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^KIV_API\s+[\w\s\*]+?\b(kiv_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = nat.load_library()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(nat.SIGNATURES), "ctypes signatures and header disagree"
    assert lib.kiv_abi_version() == 1


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(f'''
#include <stdio.h>
#include <stddef.h>
#include "{HEADER}"
#define F(T, m) printf(#T "." #m " %zu\\n", offsetof(T, m));
int main(void) {{
  printf("kiv_store %zu\\n", sizeof(kiv_store));
  printf("kiv_query %zu\\n", sizeof(kiv_query));
  printf("kiv_mask %zu\\n", sizeof(kiv_mask));
  printf("kiv_exchange %zu\\n", sizeof(kiv_exchange));
  printf("kiv_peer_rows %zu\\n", sizeof(kiv_peer_rows));
  F(kiv_store, cold_capacity) F(kiv_store, hot_capacity) F(kiv_store, cold_k) F(kiv_store, state)
  F(kiv_store, flags) F(kiv_store, page_sums)
  F(kiv_query, stride_t) F(kiv_query, scaling) F(kiv_query, top_p)
  F(kiv_mask, stride_t) F(kiv_mask, causal)
  F(kiv_exchange, arena) F(kiv_exchange, arena_bytes)
  F(kiv_peer_rows, cold_v)
  return 0;
}}''')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    out = dict(line.rsplit(" ", 1) for line in subprocess.check_output([str(exe)], text=True).split("\n") if line)
    assert int(out["kiv_store"]) == ctypes.sizeof(nat.StoreDesc)
    assert int(out["kiv_query"]) == ctypes.sizeof(nat.QueryDesc)
    assert int(out["kiv_mask"]) == ctypes.sizeof(nat.MaskDesc)
    assert int(out["kiv_exchange"]) == ctypes.sizeof(nat.ExchangeDesc)
    assert int(out["kiv_peer_rows"]) == ctypes.sizeof(nat.PeerRows)
    for key, val in out.items():
        if "." in key:
            struct, field = key.split(".")
            cls = {"kiv_store": nat.StoreDesc, "kiv_query": nat.QueryDesc, "kiv_mask": nat.MaskDesc,
                   "kiv_exchange": nat.ExchangeDesc, "kiv_peer_rows": nat.PeerRows}[struct]
            assert getattr(cls, field).offset == int(val), key


def _store(**kw):
    d = dict(batch=1, num_kv_heads=2, head_dim=64, page_size=128, dtype=1, shard_rank=0,
             shard_count=1, hot_hint=0, cold_capacity=1024, hot_capacity=0, cold_k=4096,
             cold_v=8192, summaries=12288, hot_k=None, hot_v=None, state=16384)
    d.update(kw)
    return nat.StoreDesc(**d)


def test_workspace_sizing_is_host_only():
    lib = nat.load_library()
    st = _store()
    q = nat.QueryDesc(4096, 0, 64, 64, 8, 1, 0.125, 0.0, 4, 64)
    n = lib.kiv_workspace_bytes(ctypes.byref(st), ctypes.byref(q))
    assert n > 0 and n % 256 == 0
    lay = (ctypes.c_int64 * 10)()
    assert lib.kiv_workspace_layout(ctypes.byref(st), ctypes.byref(q), lay) == 0
    offs = list(lay[:6])
    assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
    R, np_cap, u_cap, c_cap = lay[6:10]
    assert R == 8 and np_cap == 8 and u_cap == 8 and c_cap == 8 * 128 + 128


@pytest.mark.parametrize("bad", [
    dict(head_dim=6, dtype=0),          # 24-byte rows
    dict(shard_rank=2, shard_count=2),
    dict(cold_capacity=100),             # not a page multiple
    dict(cold_k=4100),                   # misaligned
    dict(state=None),
    dict(dtype=7),
])
def test_validation_rejects_before_launch(bad):
    lib = nat.load_library()
    st = _store(**bad)
    rc = lib.kiv_append_evict(ctypes.byref(st), None, None, 0, 0, 0, 0, 0, 0, None)
    assert rc in (1, 4), rc
    assert lib.kiv_last_error()


def test_null_arguments_rejected():
    lib = nat.load_library()
    assert lib.kiv_append_evict(None, None, None, 0, 0, 0, 0, 0, 0, None) == 1
    st = _store()
    q = nat.QueryDesc(None, 0, 0, 0, 8, 1, 1.0, 0.0, 4, 4)
    assert lib.kiv_coarse_select(ctypes.byref(st), ctypes.byref(q), None, 0, None, None, None) == 1
    q = nat.QueryDesc(4096, 0, 64, 64, 8, 1, 1.0, 0.0, 4, 4)
    assert lib.kiv_fine_select(ctypes.byref(st), ctypes.byref(q), None, 0, None, None, None) == 2


def test_candidate_exchange_shapes_and_peer_attention_arguments():
    """kiv_fine_exchange_supported is a host-side shape query; kiv_attend_peers
    and kiv_fine_exchange_select reject bad arguments before launching."""
    lib = nat.load_library()
    q = nat.QueryDesc(4096, 0, 64, 64, 8, 1, 0.125, 0.0, 4, 64)
    # bf16 page-sharded store with replicated summaries: eligible
    repl = _store(shard_count=2, flags=nat.STORE_REPL_SUMMARIES, page_sums=20480)
    assert lib.kiv_fine_exchange_supported(ctypes.byref(repl), ctypes.byref(q)) == 1
    # one shard, no replicated summaries, fp32 rows, or more than 16 query rows per KV head: not
    assert lib.kiv_fine_exchange_supported(ctypes.byref(_store()), ctypes.byref(q)) == 0
    plain = _store(shard_count=2)
    assert lib.kiv_fine_exchange_supported(ctypes.byref(plain), ctypes.byref(q)) == 0
    f32 = _store(shard_count=2, flags=nat.STORE_REPL_SUMMARIES, page_sums=20480, dtype=0)
    assert lib.kiv_fine_exchange_supported(ctypes.byref(f32), ctypes.byref(q)) == 0
    wide = nat.QueryDesc(4096, 0, 64, 64, 40, 1, 0.125, 0.0, 4, 64)   # 20 rows per KV head
    assert lib.kiv_fine_exchange_supported(ctypes.byref(repl), ctypes.byref(wide)) == 0
    # peer-row attention: NULL peers, one shard, or a missing peer entry are rejected
    ws_bytes = lib.kiv_workspace_bytes(ctypes.byref(repl), ctypes.byref(q))
    ws = 1 << 20
    assert lib.kiv_attend_peers(ctypes.byref(repl), ctypes.byref(q), None, ws, ws_bytes, 4096, 64, None,
                                8192, None) == 1
    peers = nat.PeerRows()
    peers.cold_k[0], peers.cold_v[0] = 4096, 8192            # own entry; shard 1 missing
    assert lib.kiv_attend_peers(ctypes.byref(repl), ctypes.byref(q), None, ws, ws_bytes, 4096, 64,
                                ctypes.byref(peers), 8192, None) == 1
    assert "shard 1" in lib.kiv_last_error().decode()
    one = _store()
    peers.cold_k[1], peers.cold_v[1] = 40960, 81920
    assert lib.kiv_attend_peers(ctypes.byref(one), ctypes.byref(q), None, ws, ws_bytes, 4096, 64,
                                ctypes.byref(peers), 8192, None) == 1
    # the candidate exchange without an exchange descriptor
    assert lib.kiv_fine_exchange_select(ctypes.byref(repl), ctypes.byref(q), ws, ws_bytes, None, 4096, None,
                                        None) == 1
