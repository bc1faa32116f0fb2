"""Load the golden fixtures written by ``tests/golden/make_golden.py``.

Inputs of the large cases are regenerated from the recorded seed with the shared
synthetic generator; small cases carry their inputs in the fixture.
"""

from __future__ import annotations

import json
import os

import numpy as np
import torch

from kiv_b200.synthetic import SynthSpec, make_problem

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASE_NAMES = ["gqa_basic", "batch2_union", "mqa", "mha_q3", "partial_only",
              "np_lt_top_pages", "p_gt_candidates", "page_boundary", "shared_reuse", "c0"]
SMALL_CASES = [c for c in CASE_NAMES if c != "c0"]


class Golden:
    def __init__(self, name: str):
        self.name = name
        z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
        self.z = {k: z[k] for k in z.files}
        self.meta = json.loads(str(self.z["meta"]))
        self.spec = SynthSpec(**self.meta["spec"])
        self.knobs = self.meta["knobs"]
        self.scaling = float(self.meta["scaling"])
        self.nq = int(self.meta["queries"])
        if "prefill_k" in self.z:
            self.prefill_k = self.z["prefill_k"]
            self.prefill_v = self.z["prefill_v"]
            self.step_k = self.z["step_k"]
            self.step_v = self.z["step_v"]
            self.queries = [self.z[f"query_{i}"] for i in range(self.nq)]
        else:
            p = make_problem(self.spec, seed=int(self.meta["seed"]), dtype=torch.float32)
            self.prefill_k = p.prefill_k.numpy()
            self.prefill_v = p.prefill_v.numpy()
            self.step_k = p.step_k.numpy()
            self.step_v = p.step_v.numpy()
            self.queries = [p.query.numpy()]

    def __getitem__(self, k):
        return self.z[k]

    def hot_mask(self):
        """Causal additive mask over hot for Q>1 (None for single-position decode)."""
        from oracle.kiv_oracle import causal_hot_mask
        Q = self.spec.query_len
        if Q == 1:
            return None
        return causal_hot_mask(self.spec.batch, Q, int(self["hot_len"]))
