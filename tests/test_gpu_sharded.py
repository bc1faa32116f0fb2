"""Page-sharded decode on 2 GPUs against the oracle and the same step on one GPU.

Two ranks (one process per GPU) build the same cache with the cold pages
sharded ``p % 2`` and run one decode layer-step through the public surface
(retrieve_indices, attend); the ranks exchange their lists and partials
through peer memory (``KIV_SHARD_EXCHANGE=peer``, the default) or the process
group's collectives.  Rank 0 also runs the step unsharded on its GPU and the
CPU oracle on the same bf16-valued inputs.  Checked on rank 0:

* every shard's page summaries cover all global pages (replicated, so the
  coarse pass needs no exchange) and equal the oracle's bit for bit;
* the sharded selection equals the oracle's except for ties within 1e-6
  relative of the top-P boundary score (fine scores of every cold token in
  float64), and the sharded attention is within 2e-2 of the float64 oracle
  over the same selection (normwise and per query row);
* the sharded and single-GPU selections are identical (same kernels, and the
  sharded merge breaks ties like the single-GPU select: score descending, id
  ascending) and their outputs agree within 1e-2 relative.

Skipped with fewer than 2 GPUs.
"""

import os
import socket
import tempfile
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
SHAPES = {
    "c2": dict(batch=1, num_query_heads=8, num_kv_heads=1, head_dim=256, cold_tokens=32768 + 77,
               hot_budget=2048, top_pages=32, top_p=512),
    "c1": dict(batch=1, num_query_heads=28, num_kv_heads=4, head_dim=128, cold_tokens=16384 + 5,
               hot_budget=1024, top_pages=16, top_p=256),
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_step(shape, dev, shard_group):
    from transformers import PretrainedConfig

    from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
    from kiv_b200.synthetic import SynthSpec, make_problem

    p = dict(SHAPES[shape])
    top_pages, top_p = p.pop("top_pages"), p.pop("top_p")
    spec = SynthSpec(**p)
    prob = make_problem(spec, seed=11, dtype=torch.bfloat16)
    cfg = KIVConfig(hot_budget=spec.hot_budget, page_size=spec.page_size, top_pages=top_pages, top_p=top_p)
    topo = ModelTopology.manual(global_layer_indices=(0,), independent_kv_layers=(0,), kv_sharing_map={},
                                num_query_heads=spec.num_query_heads, num_kv_heads=spec.num_kv_heads,
                                head_dim=spec.head_dim, num_hidden_layers=1)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, dev, shard_group=shard_group)
    t = lambda x: torch.as_tensor(x).to(dev, torch.bfloat16)
    cache.update(t(prob.prefill_k), t(prob.prefill_v), 0)
    cache.mark_prefill_complete()
    cache.update(t(prob.step_k), t(prob.step_v), 0)
    store = cache.get_cold_store(0)
    q = prob.query.to(dev)
    scaling = spec.head_dim ** -0.5
    sel, P = store.retrieve_indices(q, scaling, cfg)
    from tests.gpu_helpers import kernel_union
    # the union the fine pass built: the whole union with the candidate
    # exchange, else this shard's pages of it
    union = kernel_union(store, 1, spec.num_query_heads, 1, cfg)
    whole = shard_group is not None and any(store._fx_ok.values())
    out = store.attend(q, scaling, cfg)
    torch.cuda.synchronize(dev)
    err = store.read_state()[7]
    summ = store.page_summaries().float().cpu().numpy()
    return (sel[:, :P].cpu().numpy(), out.float().cpu().numpy(), int(err),
            (spec, prob, top_pages, top_p, summ, union, whole))


def _union_check(problem, rank):
    """The fine pass's coarse union against the oracle's union (all of it with
    the candidate exchange, else pages p % WORLD == rank), ties within 1e-6
    of a row's k-th score aside."""
    from tests.gpu_helpers import coarse_union_mismatch, oracle_decode

    spec, prob, top_pages, top_p, summ, union, whole = problem
    f32 = lambda t: t.float().numpy()
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(prob.step_k), f32(prob.step_v),
                       storage="bf16")
    np.testing.assert_array_equal(summ, ol.store.summaries)
    ref, _, sc = ol.store.coarse(f32(prob.query), spec.head_dim ** -0.5, top_pages)
    mine = np.array([p for p in ref.tolist() if whole or p % WORLD == rank], np.int64)
    k = min(top_pages, ol.store.num_pages)
    bad = coarse_union_mismatch(union, mine, sc, k)
    assert bad == [], f"rank {rank}: union pages differ from the oracle's beyond ties: {bad[:6]} " \
                      f"(kernel {len(union)} pages, oracle {len(mine)})"


def _oracle_check(sel, out, problem):
    """Sharded selection and output against the oracle (rank 0, CPU)."""
    from oracle.kiv_oracle import _group_rows, eager_attention, topk_set_mismatch
    from tests.gpu_helpers import oracle_decode, rel_err, rel_err_rows

    spec, prob, top_pages, top_p, summ, _, _ = problem
    f32 = lambda t: t.float().numpy()
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(prob.step_k), f32(prob.step_v),
                       storage="bf16")
    scaling = spec.head_dim ** -0.5
    q = f32(prob.query)
    # every shard holds the summary of every page (its own and the other shard's)
    np.testing.assert_array_equal(summ, ol.store.summaries)
    res = ol.store.retrieve_top_kv(q, scaling, top_pages, top_p)
    # fine scores of every cold token (max over heads and positions), float64
    rows = _group_rows(q.astype(np.float64), spec.num_kv_heads)
    allk = ol.store.k.astype(np.float64)
    full = (np.matmul(rows, allk.transpose(0, 1, 3, 2)) * scaling).max(axis=(1, 2))   # [B, cold]
    pos = {int(t): i for i, t in enumerate(res.cand_idx)}
    for b in range(sel.shape[0]):
        bad = topk_set_mismatch(sel[b], res.selected[b], lambda t: full[b, t], sel.shape[1],
                                res.agg_scores[b])
        assert bad == [], f"sharded selection differs from the oracle beyond ties: {bad[:4]}"
    assert sel.shape[1] == res.selected.shape[1]
    ko, vo = ol.store.gather(sel)
    ref = eager_attention(q, ko, vo, ol.hot_k, ol.hot_v, scaling)
    e, er = rel_err(out, ref), rel_err_rows(out, ref)
    assert e <= 2e-2 and er <= 2e-2, (e, er)
    return len(pos)


def _worker(rank, port, out_dir, shape, exchange):
    import datetime
    import sys

    import torch.distributed as dist

    from kiv_b200.sharding import ShardComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["KIV_SHARD_EXCHANGE"] = exchange
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    t0 = time.time()
    log = lambda msg: print(f"[rank {rank} +{time.time() - t0:.1f}s] {msg}", file=sys.stderr, flush=True)
    # the unsharded reference first, before any collective
    ref = _run_step(shape, dev, None) if rank == 0 else None
    log("single-GPU step done")
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    failure = None
    comm = ShardComm()
    try:
        sel_sh, out_sh, err_sh, problem = _run_step(shape, dev, comm)
        log("sharded step done")
        try:
            # peer exchange takes the candidate exchange (one scorer + select, no merge)
            assert problem[-1] == (exchange == "peer"), (exchange, problem[-1])
            _union_check(problem, rank)
        except AssertionError as e:
            failure = e
        if rank == 0 and failure is None:
            sel_1, out_1, err_1, _ = ref
            try:
                assert err_sh == 0 and err_1 == 0, (err_sh, err_1)
                assert sel_sh.shape == sel_1.shape, (sel_sh.shape, sel_1.shape)
                assert np.array_equal(sel_sh, sel_1), "sharded selection differs from the single-GPU selection"
                _oracle_check(sel_sh, out_sh, problem)
                log("oracle check done")
                rel = np.abs(out_sh - out_1).max() / max(np.abs(out_1).max(), 1e-30)
                assert rel <= 1e-2, rel
                with open(os.path.join(out_dir, "ok"), "w") as f:
                    f.write(f"{rel}")
            except AssertionError as e:
                failure = e
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()
    if failure is not None:
        raise failure


@pytest.mark.parametrize("exchange", ["peer", "collective"])
@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_sharded_step_matches_single_gpu(shape, exchange):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_worker, args=(_free_port(), d, shape, exchange), nprocs=WORLD, join=False,
                                 start_method="spawn")
        deadline = time.time() + 300
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("sharded ranks did not finish in 300 s")
        assert os.path.exists(os.path.join(d, "ok"))


SEQ_SHAPE = dict(batch=4, num_query_heads=32, num_kv_heads=8, head_dim=128, cold_tokens=8192 + 37,
                 hot_budget=512)


def _seq_worker(rank, port, out_dir):
    """Sequence sharding: rank r holds sequences [2r, 2r + 2) of a batch of 4;
    its selection and attention must match the unsharded oracle's for them
    (the page union spans all four sequences, OR-reduced over the ranks)."""
    import datetime

    import torch.distributed as dist
    from transformers import PretrainedConfig

    from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
    from kiv_b200.synthetic import SynthSpec, make_problem
    from oracle.kiv_oracle import eager_attention, topk_set_mismatch
    from tests.gpu_helpers import oracle_decode, rel_err, rel_err_rows

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        spec = SynthSpec(**SEQ_SHAPE)
        top_pages, top_p = 8, 256
        prob = make_problem(spec, seed=13, dtype=torch.bfloat16)
        lo, hi = 2 * rank, 2 * rank + 2
        cfg = KIVConfig(hot_budget=spec.hot_budget, page_size=spec.page_size, top_pages=top_pages, top_p=top_p,
                        telemetry=False)
        topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=spec.num_query_heads,
                                    num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim, num_hidden_layers=1)
        cache = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, dev, batch_group=dist.group.WORLD)
        t = lambda x: x[lo:hi].to(dev)
        cache.update(t(prob.prefill_k), t(prob.prefill_v), 0)
        cache.mark_prefill_complete()
        cache.update(t(prob.step_k), t(prob.step_v), 0)
        store = cache.get_cold_store(0)
        q = t(prob.query)
        scaling = spec.head_dim ** -0.5
        sel, P = store.retrieve_indices(q, scaling, cfg)
        out = store.attend(q, scaling, cfg).float().cpu().numpy()
        assert store.read_state()[7] == 0
        f32 = lambda x: x.float().numpy()
        ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(prob.step_k), f32(prob.step_v),
                           storage="bf16")
        res = ol.store.retrieve_top_kv(f32(prob.query), scaling, top_pages, top_p)
        got = sel[:, :P].cpu().numpy()
        assert P == res.selected.shape[1]
        pos = {int(c): i for i, c in enumerate(res.cand_idx)}
        for j, b in enumerate(range(lo, hi)):
            bad = topk_set_mismatch(got[j], res.selected[b], lambda c: res.agg_scores[b, pos[c]], P,
                                    res.agg_scores[b])
            assert bad == [], f"sequence {b}: selection differs beyond ties: {bad[:4]}"
        ko, vo = ol.store.gather(np.concatenate([np.zeros((lo, P), np.int64), got,
                                                 np.zeros((spec.batch - hi, P), np.int64)]))
        ref = eager_attention(f32(prob.query), ko, vo, ol.hot_k, ol.hot_v, scaling)[lo:hi]
        assert rel_err(out, ref) <= 2e-2 and rel_err_rows(out, ref) <= 2e-2
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("ok")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_step_matches_oracle():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_seq_worker, args=(_free_port(), d), nprocs=WORLD, join=False,
                                 start_method="spawn")
        deadline = time.time() + 300
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("sequence-sharded ranks did not finish in 300 s")
        assert all(os.path.exists(os.path.join(d, f"ok{r}")) for r in range(WORLD))


def _persist_worker(rank, port, out_dir):
    """Page-sharded save and resume: every rank saves its store, a fresh sharded
    cache loads the files, and the next decode step gives the same selection
    and output on both caches."""
    import datetime

    import torch.distributed as dist
    from transformers import PretrainedConfig

    from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
    from kiv_b200.sharding import ShardComm
    from kiv_b200.synthetic import SynthSpec, make_problem

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    comm = ShardComm()
    try:
        spec = SynthSpec(batch=1, num_query_heads=8, num_kv_heads=1, head_dim=256, cold_tokens=20480 + 45,
                         hot_budget=512)
        prob = make_problem(spec, seed=23, dtype=torch.bfloat16)
        cfg = KIVConfig(hot_budget=spec.hot_budget, page_size=128, top_pages=16, top_p=256, telemetry=False)
        topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=8, num_kv_heads=1, head_dim=256,
                                    num_hidden_layers=1)
        mk = lambda: TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, dev, shard_group=comm)
        a = mk()
        a.update(prob.prefill_k.to(dev), prob.prefill_v.to(dev), 0)
        a.mark_prefill_complete()
        a.update(prob.step_k.to(dev), prob.step_v.to(dev), 0)
        d = os.path.join(out_dir, "ckpt")
        if rank == 0:
            os.makedirs(d, exist_ok=True)
        dist.barrier()
        a.save(d)
        dist.barrier()
        b = mk()
        b.load(d)
        g = torch.Generator().manual_seed(3)
        q = torch.randn(1, 8, 1, 256, generator=g).to(dev, torch.bfloat16)
        k = (0.3 * torch.randn(1, 1, 1, 256, generator=g)).to(dev, torch.bfloat16)
        v = torch.randn(1, 1, 1, 256, generator=g).to(dev, torch.bfloat16)
        res = []
        for c in (a, b):
            c.update(k, v, 0)
            st = c.get_cold_store(0)
            sel, P = st.retrieve_indices(q, 256 ** -0.5, cfg)
            out = st.attend(q, 256 ** -0.5, cfg)
            torch.cuda.synchronize(dev)
            assert st.read_state()[7] == 0
            res.append((sel[:, :P].cpu(), out.float().cpu(), st.page_summaries().cpu()))
        assert torch.equal(res[0][0], res[1][0]), "selection differs after resume"
        assert torch.equal(res[0][1], res[1][1]), "output differs after resume"
        assert torch.equal(res[0][2], res[1][2]), "summaries differ after resume"
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("ok")
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()


def test_page_sharded_save_and_resume():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_persist_worker, args=(_free_port(), d), nprocs=WORLD, join=False,
                                 start_method="spawn")
        deadline = time.time() + 300
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("ranks did not finish in 300 s")
        assert all(os.path.exists(os.path.join(d, f"ok{r}")) for r in range(WORLD))


def _steps_worker(rank, port, out_dir):
    """Many decode steps of a batch-2 page-sharded cache (peer transport:
    candidate exchange + peer-row attention) against the same steps on one GPU:
    pages complete on the way (running page sums, summaries), both exchange
    parities and many epochs are used."""
    import datetime

    import torch.distributed as dist
    from transformers import PretrainedConfig

    from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
    from kiv_b200.sharding import ShardComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["KIV_SHARD_EXCHANGE"] = "peer"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    B, HQ, HKV, D, PRE, STEPS = 2, 8, 2, 128, 4096 + 60, 140
    cfg = KIVConfig(hot_budget=256, page_size=128, top_pages=8, top_p=128, telemetry=False)
    topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=HQ, num_kv_heads=HKV, head_dim=D,
                                num_hidden_layers=1)
    g = torch.Generator().manual_seed(31)
    pre_k = torch.randn(B, HKV, PRE, D, generator=g).to(torch.bfloat16)
    pre_v = torch.randn(B, HKV, PRE, D, generator=g).to(torch.bfloat16)
    ks = torch.randn(STEPS, B, HKV, 1, D, generator=g).to(torch.bfloat16)
    vs = torch.randn(STEPS, B, HKV, 1, D, generator=g).to(torch.bfloat16)
    qs = torch.randn(STEPS, B, HQ, 1, D, generator=g).to(torch.bfloat16)
    scaling = D ** -0.5

    def build(group):
        c = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, dev, shard_group=group)
        c.update(pre_k.to(dev), pre_v.to(dev), 0)
        c.mark_prefill_complete()
        return c

    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    comm = ShardComm()
    try:
        single = build(None) if rank == 0 else None
        sharded = build(comm)
        pages0 = sharded.get_cold_store(0).num_pages
        worst = 0.0
        for s in range(STEPS):
            outs = []
            for c in ([sharded, single] if rank == 0 else [sharded]):
                c.update(ks[s].to(dev), vs[s].to(dev), 0)
                st = c.get_cold_store(0)
                sel, P = st.retrieve_indices(qs[s].to(dev), scaling, cfg)
                out = st.attend(qs[s].to(dev), scaling, cfg)
                outs.append((sel[:, :P].cpu(), out.float().cpu(), st))
            if rank == 0:
                (s_sel, s_out, s_st), (o_sel, o_out, o_st) = outs
                assert s_st.read_state()[7] == 0 and o_st.read_state()[7] == 0, f"step {s}: error bits"
                assert torch.equal(s_sel, o_sel), f"step {s}: sharded selection differs from one GPU"
                rel = float((s_out - o_out).abs().max() / o_out.abs().max().clamp_min(1e-30))
                worst = max(worst, rel)
                assert rel <= 1e-2, f"step {s}: output rel {rel}"
        assert any(sharded.get_cold_store(0)._fx_ok.values()), "the candidate exchange did not run"
        assert sharded.get_cold_store(0).num_pages > pages0, "no page completed during the steps"
        if rank == 0:
            with open(os.path.join(out_dir, "ok"), "w") as f:
                f.write(f"{worst}")
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()


def test_sharded_decode_steps_match_single_gpu():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_steps_worker, args=(_free_port(), d), nprocs=WORLD, join=False,
                                 start_method="spawn")
        deadline = time.time() + 300
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("ranks did not finish in 300 s")
        assert os.path.exists(os.path.join(d, "ok"))
