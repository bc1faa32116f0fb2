"""On-disk format of a cold store, for resuming a sequence later.

The reference keeps no state on disk; this is the page-store persistence of
the host overflow tier's row in the build plan.  One file per independent KV
layer, little-endian:

    bytes 0-7     magic b"KIVSTOR1"
    bytes 8-15    u64: length H of the header
    bytes 16..    UTF-8 JSON header (H bytes), zero padding to 64 bytes
    data blocks   at the offsets the header lists, each 64-byte aligned:
                    cold_k, cold_v  [B, Hkv, cold_len, D]  cold rows in token order
                    hot_k, hot_v    [B, Hkv, hot_len, D]   hot window, oldest first

Header keys: format, version, batch, num_kv_heads, head_dim, page_size, dtype,
cold_len, hot_len, blocks ({name: [offset, nbytes]}) and an optional "meta"
dict of the caller.  Page summaries are not stored: loading replays the cold
rows through the eviction kernel, which rebuilds them bit for bit, and the
rows land in whichever tier (HBM ring or pinned host memory) the loading
store's configuration puts them.

A page-sharded store (one process per GPU) is saved rank by rank: each rank's
file holds the rows of its own pages in local page order (``cold_k``,
``cold_v`` [B, Hkv, local_rows, D]), the replicated hot window, every global
page's summary (``summaries`` [B, Hkv, pages, D]) and the running sums of the
page being filled (``page_sums`` fp32 [2, B, Hkv, D]); the header adds a
``shard`` entry {rank, count, local_rows, page_sum_slot}.  Such a file loads
into an empty store of the same rank and shard count by plain copies (the
other ranks' rows, which rebuilt summaries would need, are not on this rank).
"""

from __future__ import annotations

import json
import math
import os
import struct

import torch

from . import _native as nat

MAGIC = b"KIVSTOR1"
VERSION = 1
_ALIGN = 64
_DTYPES = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}
_FROM_NAME = {v: k for k, v in _DTYPES.items()}


def _pad(n: int) -> int:
    return (-n) % _ALIGN


def _cold_rows(store) -> tuple[torch.Tensor, torch.Tensor]:
    """The store's cold rows [B, Hkv, cold_len, D] in token order (on the CPU)."""
    n, S = store.cold_length, store._page_size
    if n == 0:
        shape = (store._batch, store._num_kv_heads, 0, store._head_dim)
        return torch.empty(shape, dtype=store._dtype), torch.empty(shape, dtype=store._dtype)
    if not store.tiered:
        return store._k[:, :, :n].cpu(), store._v[:, :, :n].cpu()
    started = math.ceil(n / S)
    R = store._ring_pages
    thr = max(0, started - R)              # pages below this live in the host tier
    parts_k = [store._host_k[:, :, :thr * S].clone()]
    parts_v = [store._host_v[:, :, :thr * S].clone()]
    idx = torch.cat([torch.arange(S) + (lp % R) * S for lp in range(thr, started)])[:n - thr * S]
    idx = idx.to(store.device)
    parts_k.append(store._k[:, :, idx].cpu())
    parts_v.append(store._v[:, :, idx].cpu())
    return torch.cat(parts_k, dim=2), torch.cat(parts_v, dim=2)


def _local_rows(store) -> int:
    """Rows of a page-sharded store's own pages (a prefix of its token slots)."""
    S, N, r = store._page_size, store._shard_count, store._shard_rank
    full = store._local_pages(store.num_pages) * S
    part = store._partial_len if store.num_pages % N == r else 0
    return full + part


def save_store(store, path: str, meta: dict | None = None) -> dict:
    """Write one store to `path`; returns the header."""
    if store._state is None:
        raise RuntimeError("the store holds nothing yet")
    if store.device.type == "cuda":
        torch.cuda.synchronize(store.device)
    hk, hv = store.hot_keys().cpu(), store.hot_values().cpu()
    header = {"format": "kiv_b200 cold store", "version": VERSION, "batch": store._batch,
              "num_kv_heads": store._num_kv_heads, "head_dim": store._head_dim,
              "page_size": store._page_size, "dtype": _DTYPES[store._dtype],
              "cold_len": store.cold_length, "hot_len": store.hot_length, "meta": meta or {}}
    if store._shard_count == 1:
        ck, cv = _cold_rows(store)
        blobs = {"cold_k": ck, "cold_v": cv, "hot_k": hk, "hot_v": hv}
    else:
        if not store.replicated_summaries:
            raise NotImplementedError("page-sharded stores with a host tier are not saved")
        n = _local_rows(store)
        words = store.read_state()
        blobs = {"cold_k": store._k[:, :, :n].cpu(), "cold_v": store._v[:, :, :n].cpu(), "hot_k": hk,
                 "hot_v": hv, "summaries": store.page_summaries().cpu(),
                 "page_sums": store._page_sums.cpu()}
        header["shard"] = {"rank": store._shard_rank, "count": store._shard_count, "local_rows": n,
                           "page_sum_slot": int(words[nat.ST_PAGESUM_SLOT]) & 1}
    # offsets depend on the header length: fix the block table with a first pass
    blocks = {name: [0, t.numel() * t.element_size()] for name, t in blobs.items()}
    prev = None
    while True:
        header["blocks"] = blocks
        hb = json.dumps(header, sort_keys=True).encode()
        if len(hb) == prev:
            break
        prev = len(hb)
        off = 16 + len(hb) + _pad(16 + len(hb))
        for name in blobs:
            blocks[name] = [off, blocks[name][1]]
            off += blocks[name][1] + _pad(blocks[name][1])
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        f.write(b"\0" * _pad(16 + len(hb)))
        for name, t in blobs.items():
            assert f.tell() == blocks[name][0]
            raw = t.contiguous().view(torch.uint8).numpy().tobytes()
            f.write(raw)
            f.write(b"\0" * _pad(len(raw)))
    os.replace(tmp, path)
    return header


def read_header(path: str) -> dict:
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path}: not a kiv_b200 store file")
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n).decode())
    if header.get("version") != VERSION:
        raise ValueError(f"{path}: unsupported store file version {header.get('version')}")
    return header


def _read_block(path: str, header: dict, name: str, shape: tuple) -> torch.Tensor:
    off, nbytes = header["blocks"][name]
    dt = torch.float32 if name == "page_sums" else _FROM_NAME[header["dtype"]]
    with open(path, "rb") as f:
        f.seek(off)
        raw = bytearray(f.read(nbytes))
    if len(raw) != nbytes:
        raise ValueError(f"{path}: block {name} truncated")
    return torch.frombuffer(raw, dtype=torch.uint8).view(dt).view(shape)


def load_store(store, path: str, chunk: int = 65536) -> dict:
    """Fill an empty store from `path`: cold rows through the eviction kernel
    (summaries rebuilt), then the hot window.  Returns the header."""
    header = read_header(path)
    if store._state is not None and (store.cold_length or store.hot_length):
        raise RuntimeError("load_store needs an empty store")
    shard = header.get("shard")
    mine = (getattr(store, "_shard_rank", 0), store._shard_count)
    if (shard is None) != (mine[1] == 1) or (shard is not None and (shard["rank"], shard["count"]) != mine):
        raise ValueError(f"{path}: saved for shard {shard and (shard['rank'], shard['count'])}, the store is "
                         f"shard {mine}")
    geo = (store._num_kv_heads, store._head_dim, store._page_size)
    if (header["num_kv_heads"], header["head_dim"], header["page_size"]) != geo:
        raise ValueError(f"{path}: store geometry {header['num_kv_heads'], header['head_dim'], header['page_size']}"
                         f" does not match {geo}")
    B, H, D = header["batch"], header["num_kv_heads"], header["head_dim"]
    n, h = header["cold_len"], header["hot_len"]
    if shard is not None:
        _load_shard(store, path, header, B, H, D)
        if h > 0:
            store.set_hot(_read_block(path, header, "hot_k", (B, H, h, D)).to(store.device),
                          _read_block(path, header, "hot_v", (B, H, h, D)).to(store.device))
        if store.device.type == "cuda":
            torch.cuda.synchronize(store.device)
        return header
    ck = _read_block(path, header, "cold_k", (B, H, n, D))
    cv = _read_block(path, header, "cold_v", (B, H, n, D))
    for a in range(0, n, chunk):
        store.evict_from_hot(ck[:, :, a:a + chunk].to(store.device), cv[:, :, a:a + chunk].to(store.device))
    if h > 0:
        store.set_hot(_read_block(path, header, "hot_k", (B, H, h, D)).to(store.device),
                      _read_block(path, header, "hot_v", (B, H, h, D)).to(store.device))
    if store.device.type == "cuda":
        torch.cuda.synchronize(store.device)
    return header


def _load_shard(store, path: str, header: dict, B: int, H: int, D: int) -> None:
    """A page-sharded store's own rows, every page's summary and the running page
    sums, copied into place; the device state gets the global cold length."""
    sh = header["shard"]
    n, local = header["cold_len"], sh["local_rows"]
    dt = _FROM_NAME[header["dtype"]]
    store._ensure_alloc(B, dt)
    store.reserve(n)
    pages = n // store._page_size
    if local:
        store._k[:, :, :local].copy_(_read_block(path, header, "cold_k", (B, H, local, D)).to(store.device))
        store._v[:, :, :local].copy_(_read_block(path, header, "cold_v", (B, H, local, D)).to(store.device))
    if pages:
        store._summ[:, :, :pages].copy_(_read_block(path, header, "summaries", (B, H, pages, D)).to(store.device))
    store._page_sums.copy_(_read_block(path, header, "page_sums", (2, B, H, D)).to(store.device))
    store._state[nat.ST_COLD_LEN].fill_(n)
    store._state[nat.ST_PAGESUM_SLOT].fill_(sh["page_sum_slot"])
    store._cold_len = n
