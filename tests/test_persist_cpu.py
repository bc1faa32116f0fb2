"""The on-disk store format on CPU: header, 64-byte aligned blocks, round trip
of the rows through save_store / load_store (with stand-in stores: the real
store is a CUDA object), and the checks on load."""

import struct
from types import SimpleNamespace

import pytest
import torch

from kiv_b200 import persist


class _Saved(SimpleNamespace):
    """What save_store reads from a store."""

    def hot_keys(self):
        return self.hk

    def hot_values(self):
        return self.hv


class _Loading:
    """Records what load_store hands to a store."""

    def __init__(self, H=2, D=16, S=8):
        self._shard_count, self._state = 1, None
        self._num_kv_heads, self._head_dim, self._page_size = H, D, S
        self.device = torch.device("cpu")
        self.cold_k, self.cold_v, self.hot = [], [], None
        self.cold_length = self.hot_length = 0

    def evict_from_hot(self, k, v):
        self.cold_k.append(k.clone())
        self.cold_v.append(v.clone())

    def set_hot(self, k, v):
        self.hot = (k.clone(), v.clone())


def _saved(dtype, n=37, h=5, B=2, H=2, D=16, S=8):
    g = torch.Generator().manual_seed(0)
    mk = lambda t: torch.randn(B, H, t, D, generator=g).to(dtype)
    return _Saved(_shard_count=1, _state=object(), _batch=B, _num_kv_heads=H, _head_dim=D, _page_size=S,
                  _dtype=dtype, cold_length=n, hot_length=h, tiered=False, device=torch.device("cpu"),
                  _k=mk(n + 11), _v=mk(n + 11), hk=mk(h), hv=mk(h))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_round_trip_and_layout(tmp_path, dtype):
    st = _saved(dtype)
    path = str(tmp_path / "s.kivstore")
    hdr = persist.save_store(st, path, meta={"layer": 3})
    raw = open(path, "rb").read()
    assert raw[:8] == persist.MAGIC
    (hl,) = struct.unpack("<Q", raw[8:16])
    assert persist.read_header(path) == hdr and hdr["meta"] == {"layer": 3}
    for name, (off, nb) in hdr["blocks"].items():
        assert off % 64 == 0 and off >= 16 + hl
    ld = _Loading()
    persist.load_store(ld, path, chunk=10)
    assert [k.shape[2] for k in ld.cold_k] == [10, 10, 10, 7]
    assert torch.equal(torch.cat(ld.cold_k, 2), st._k[:, :, :37]) and torch.equal(torch.cat(ld.cold_v, 2), st._v[:, :, :37])
    assert torch.equal(ld.hot[0], st.hk) and torch.equal(ld.hot[1], st.hv)


def test_load_rejects_bad_files(tmp_path):
    p = tmp_path / "x.kivstore"
    p.write_bytes(b"NOTASTORE" + b"\0" * 32)
    with pytest.raises(ValueError):
        persist.read_header(str(p))
    st = _saved(torch.bfloat16)
    persist.save_store(st, str(p))
    with pytest.raises(ValueError):
        persist.load_store(_Loading(D=32), str(p))          # geometry mismatch
    busy = _Loading()
    busy._state, busy.cold_length = object(), 5
    with pytest.raises(RuntimeError):
        persist.load_store(busy, str(p))                   # not empty
    sharded = _saved(torch.bfloat16)
    sharded._shard_count = 2
    sharded.replicated_summaries = False        # page-sharded with a host tier
    with pytest.raises(NotImplementedError):
        persist.save_store(sharded, str(tmp_path / "y.kivstore"))


def test_config_host_tier_validation():
    from kiv_b200 import KIVConfig
    with pytest.raises(ValueError):
        KIVConfig(host_tokens=1024)                       # needs the ring size
    with pytest.raises(ValueError):
        KIVConfig(cold_capacity=1024, host_tokens=1024, stage_pages=0)
    assert KIVConfig(cold_capacity=1024, host_tokens=4096).stage_pages == 1024


class _ShardSaved(_Saved):
    """A page-sharded store as save_store reads it (stand-in, CPU tensors)."""

    replicated_summaries = True

    def _local_pages(self, n):
        r, c = self._shard_rank, self._shard_count
        return (n - r + c - 1) // c if n > r else 0

    @property
    def num_pages(self):
        return self.cold_length // self._page_size

    @property
    def _partial_len(self):
        return self.cold_length % self._page_size

    def read_state(self):
        return self.words

    def page_summaries(self):
        return self.summ[:, :, :self.num_pages]


class _ShardLoading:
    """A fresh page-sharded store for load_store: records what is copied in."""

    def __init__(self, rank, count, B=2, H=2, D=16, S=8, slots=64, dtype=torch.bfloat16):
        self._shard_rank, self._shard_count = rank, count
        self._num_kv_heads, self._head_dim, self._page_size = H, D, S
        self.device = torch.device("cpu")
        self._state = torch.zeros(32, dtype=torch.int64)
        self._k = torch.zeros(B, H, slots, D, dtype=dtype)
        self._v = torch.zeros_like(self._k)
        self._summ = torch.zeros(B, H, count * slots // S, D, dtype=dtype)
        self._page_sums = torch.zeros(2, B, H, D)
        self.cold_length = self.hot_length = 0
        self.hot = None

    def _ensure_alloc(self, B, dtype):
        assert B == self._k.shape[0] and dtype == self._k.dtype

    def reserve(self, n):
        assert n <= self._k.shape[2] * self._shard_count

    def set_hot(self, k, v):
        self.hot = (k.clone(), v.clone())


def test_page_sharded_store_round_trip(tmp_path):
    """Rank 1 of 2: its own rows (a prefix of its slots), all summaries, the
    running page sums and the page-sum slot come back by plain copies; a file
    of another rank or of an unsharded store is refused."""
    B, H, D, S, n, h = 2, 2, 16, 8, 8 * 9 + 5, 3
    g = torch.Generator().manual_seed(1)
    mk = lambda *sh: torch.randn(*sh, generator=g).to(torch.bfloat16)
    # 9 full pages + a partial one: rank 1 owns pages 1, 3, 5, 7 and the partial page 9
    local = 4 * S + 5
    words = [0] * 32
    words[21] = 1
    st = _ShardSaved(_shard_count=2, _shard_rank=1, _state=object(), _batch=B, _num_kv_heads=H, _head_dim=D,
                     _page_size=S, _dtype=torch.bfloat16, cold_length=n, hot_length=h, tiered=False,
                     device=torch.device("cpu"), _k=mk(B, H, 64, D), _v=mk(B, H, 64, D), hk=mk(B, H, h, D),
                     hv=mk(B, H, h, D), summ=mk(B, H, 16, D), _page_sums=torch.randn(2, B, H, D, generator=g),
                     words=words)
    path = str(tmp_path / "r1.kivstore")
    hdr = persist.save_store(st, path)
    assert hdr["shard"] == {"rank": 1, "count": 2, "local_rows": local, "page_sum_slot": 1}
    dst = _ShardLoading(1, 2)
    persist.load_store(dst, path)
    assert torch.equal(dst._k[:, :, :local], st._k[:, :, :local])
    assert torch.equal(dst._v[:, :, :local], st._v[:, :, :local])
    assert torch.equal(dst._summ[:, :, :n // S], st.summ[:, :, :n // S])
    assert torch.equal(dst._page_sums, st._page_sums)
    assert int(dst._state[0]) == n and int(dst._state[21]) == 1 and dst._cold_len == n
    assert torch.equal(dst.hot[0], st.hk) and torch.equal(dst.hot[1], st.hv)
    with pytest.raises(ValueError, match="shard"):
        persist.load_store(_ShardLoading(0, 2), path)
    with pytest.raises(ValueError, match="shard"):
        persist.load_store(_Loading(), path)
