"""The PyTorch operator library (``torch.ops.kiv.*``) on the CPU: it loads, every
compute entry point of the C ABI is registered with a schema that declares
what it writes, the Meta kernels let a decode step be traced with fake CUDA
tensors, and the shape-only workspace query agrees with the C ABI's."""

import ctypes

import torch
from torch.fx.experimental.proxy_tensor import make_fx
from torch._subclasses.fake_tensor import FakeTensorMode

from kiv_b200 import _native as nat
from kiv_b200 import ops


def test_every_operator_is_registered():
    K = ops.kiv()
    for name in ops.OP_NAMES:
        assert hasattr(K, name), name
    # writers declare their mutations; the store list is always (a!)
    for name in ops.OP_NAMES:
        sch = str(getattr(K, name).default._schema)
        if name in ("workspace_layout", "gather_rows", "attend_merge"):
            assert "Tensor[] store" in sch, sch
        else:
            assert "Tensor(a!)[] store" in sch, sch
    assert "Tensor(d!) out" in str(K.retrieve_attend.default._schema)
    assert "Tensor(c!)? out" in str(K.attend.default._schema)


def _fake_store(dev, D=64, H=2, cold=4096, hot=512, dtype=torch.bfloat16):
    ck = torch.empty(1, H, cold, D, dtype=dtype, device=dev)
    cv = torch.empty_like(ck)
    sm = torch.empty(1, H, cold // 128, D, dtype=dtype, device=dev)
    hk = torch.empty(1, H, hot, D, dtype=dtype, device=dev)
    hv = torch.empty_like(hk)
    st = torch.zeros(32, dtype=torch.int64, device=dev)
    e = torch.empty(0, dtype=dtype, device=dev)
    return [ck, cv, sm, hk, hv, st, e, e, torch.empty(0, device=dev)], [128, 0, 1, hot, 0, 0]


def test_decode_step_traces_with_fake_tensors():
    dev = torch.device("cuda")

    def step(store, q, ws, sel, out, knew, vnew):
        geom = [128, 0, 1, 512, 0, 0]
        torch.ops.kiv.append_evict(store, geom, knew, vnew, 512, 1)
        torch.ops.kiv.coarse_select(store, geom, q, 0.125, 8, 128, 0.0, ws, None, None)
        torch.ops.kiv.fine_select(store, geom, q, 0.125, 8, 128, 0.0, ws, sel, None)
        torch.ops.kiv.attend(store, geom, q, 0.125, 8, 128, 0.0, ws, sel, None, False, 0, 1, out, None)
        return out

    ops.load()
    with FakeTensorMode():
        store, geom = _fake_store(dev)
        q = torch.empty(1, 8, 1, 64, dtype=torch.bfloat16, device=dev)
        lay = torch.ops.kiv.workspace_layout(store, geom, q, 8, 128)
        ws = torch.empty(lay[10], dtype=torch.uint8, device=dev)
        sel = torch.empty(1, 128, dtype=torch.int32, device=dev)
        out = torch.empty(1, 1, 8, 64, dtype=torch.bfloat16, device=dev)
        kn = torch.empty(1, 2, 1, 64, dtype=torch.bfloat16, device=dev)
        gm = make_fx(step, tracing_mode="fake")(store, q, ws, sel, out, kn, kn.clone())
    code = gm.code
    for name in ("append_evict", "coarse_select", "fine_select", "attend"):
        assert f"torch.ops.kiv.{name}.default" in code, name


def test_workspace_layout_matches_the_c_abi():
    L = nat.load_library()
    for dtype, D, H, Hq, Q, tp, tpp in ((torch.bfloat16, 256, 1, 8, 1, 64, 1024),
                                        (torch.float32, 64, 4, 32, 1, 32, 256),
                                        (torch.bfloat16, 128, 4, 28, 3, 32, 512)):
        store, geom = _fake_store(torch.device("meta"), D=D, H=H, cold=65536, hot=2048, dtype=dtype)
        q = torch.empty(1, Hq, Q, D, dtype=dtype, device="meta")
        lay = ops.kiv().workspace_layout(store, geom, q, tp, tpp)
        fake = 1 << 20
        sd = nat.StoreDesc(1, H, D, 128, nat.KIV_DTYPE[dtype], 0, 1, 2048, 65536, 2048, fake, fake, fake, fake,
                           fake, fake, 0, None, None, 0, 0)
        qd = nat.QueryDesc(fake, Hq * Q * D, Q * D, D, Hq, Q, 1.0, 0.0, tp, tpp)
        want = (ctypes.c_int64 * 10)()
        nat.check(L.kiv_workspace_layout(ctypes.byref(sd), ctypes.byref(qd), want), "layout")
        assert list(lay[:10]) == list(want)
        assert lay[10] == L.kiv_workspace_bytes(ctypes.byref(sd), ctypes.byref(qd))


def test_operator_errors_raise_not_crash():
    """A shape the library rejects comes back as KIVNativeError with its message."""
    import pytest

    store, geom = _fake_store(torch.device("meta"), D=6, dtype=torch.float32)
    q = torch.empty(1, 4, 1, 6, device="meta")
    with pytest.raises(nat.KIVNativeError, match="multiple of 16 bytes"):
        ops.call(ops.kiv().workspace_layout, store, geom, q, 4, 16)
