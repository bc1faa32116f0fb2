"""Kernel timelines of a decode layer-step: an instrumented copy of the package
(``python -m kiv_b200.timeline.build --out DIR``) and probes, run as scripts
so that they import the copy, that replay a layer-step and print, per stamp,
the earliest and latest CTA (``kiv_b200/timeline/probe.py`` on one GPU,
``kiv_b200/timeline/probe_shard.py`` under ``torch.distributed.run``).  Development tooling; the product path never
imports it."""
