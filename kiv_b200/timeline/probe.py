"""Timeline of replayed decode layer-steps on one GPU, from an instrumented copy.

    python -m kiv_b200.timeline.build --out DIR
    python kiv_b200/timeline/probe.py --pkg DIR [--workload c2]

Builds the workload with 2 layers in a ``DecodeGraph``, replays it, and for
each stamp prints the earliest and latest CTA (µs after layer 1's eviction
passed its dependency wait), median of 30 replays.
"""
import argparse
import os
import sys

NAMES = {0: "evict wait", 1: "evict end", 2: "coarse scorer wait", 3: "coarse scorer end", 4: "top-k wait",
         5: "top-k staged", 9: "top-k end", 10: "fine scorer wait", 11: "fine union built", 12: "fine scorer end",
         13: "fine select wait", 14: "fine select end", 17: "fine exchange wait", 18: "fine lists in",
         19: "fine exchange end", 15: "attention cold wait", 16: "attention end", 20: "partials exchange wait",
         21: "partials in", 22: "partials exchange end", 23: "candidates in (exchange)"}


def load(pkg):
    """Import the instrumented copy (before anything imports the product package)."""
    sys.path.insert(0, os.path.abspath(pkg))
    import kiv_b200
    if not kiv_b200.__file__.startswith(os.path.abspath(pkg)):
        raise SystemExit(f"kiv_b200 imported from {kiv_b200.__file__}, not from {pkg}")
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(1, root)


def run(cache, layers, w, q, k, v, dev, barrier=lambda: None, replays=30):
    import numpy as np
    import torch

    from kiv_b200.decode_graph import DecodeGraph

    sq, sk, sv = q[0].clone(), k[0].clone(), v[0].clone()
    out = torch.empty(layers, w.get("batch", 1), 1, w["hq"], w["d"], dtype=torch.bfloat16, device=dev)
    g = DecodeGraph(cache, list(range(layers)), w["d"] ** -0.5, sq, sk, sv, out, max_steps=replays + 16)
    st = cache.get_cold_store(layers - 1)._state
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    barrier()
    rows = []
    for i in range(replays):
        sq.copy_(q[i % q.shape[0]]); sk.copy_(k[i % k.shape[0]]); sv.copy_(v[i % v.shape[0]])
        st[32::2] = np.iinfo(np.int64).max
        st[33::2] = 0
        torch.cuda.synchronize()
        barrier()
        g.replay()
        torch.cuda.synchronize()
        rows.append(st.cpu().numpy().copy())
    R = np.array(rows)
    t0 = R[:, 32].astype(np.float64)
    med = {}
    for s in NAMES:
        lo, hi = R[:, 32 + 2 * s].astype(np.float64), R[:, 33 + 2 * s].astype(np.float64)
        ok = hi > 0
        if ok.sum():
            med[s] = (float(np.median((lo - t0)[ok]) / 1e3), float(np.median((hi - t0)[ok]) / 1e3))
    return med, g


def table(meds, title):
    print(title)
    print("slot stamp                    " + "  ".join(f"r{r} first    last" for r in range(len(meds))))
    for s, name in sorted(NAMES.items(), key=lambda kv: meds[0].get(kv[0], (1e9,))[0]):
        if s in meds[0]:
            print(f"{s:4d} {name:24s}" + "  ".join(f"{m[s][0]:8.2f} {m[s][1]:7.2f}" for m in meds))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--pkg", required=True)
    ap.add_argument("--workload", default="c2")
    a = ap.parse_args()
    load(a.pkg)
    import torch

    import bench
    from kiv_b200 import KIVConfig

    w = dict(bench.WORKLOADS[a.workload])
    w["layers"] = 2
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    kcfg = KIVConfig(hot_budget=w["hot"], top_p=w["top_p"], page_size=128, top_pages=w["top_pages"],
                     cold_capacity=w["cold"] + w["hot"] + 4096, hot_slack=4096, telemetry=False)
    q, k, v = bench.make_inputs(w, dev, 64)
    cache = bench.build_cache(w, dev, kcfg, None, q[0, :, :, :, 0, :])
    med, _ = run(cache, 2, w, q, k, v, dev)
    table([med], f"{a.workload} on 1 GPU: earliest / latest CTA per stamp, µs after the eviction's wait "
                 "(median of 30 replays)")


if __name__ == "__main__":
    main()
