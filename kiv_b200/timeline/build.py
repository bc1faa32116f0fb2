"""Build an instrumented copy of the package: %globaltimer stamps at the
anchors a stamp file names, written into state words 32.. of each store.

    python -m kiv_b200.timeline.build --out DIR [--stamps FILE]

copies ``kiv_b200/`` and ``include/`` to DIR, widens the device state to 160
words there, inserts ``TL(slot)`` (thread 0 of each CTA: atomic min and max of
the time into words 32 + 2*slot and 33 + 2*slot) after each anchor, and builds
the copy with its Makefile.  The product build carries no stamps; the probes
in this directory import the copy.  Stamp file lines:
``file ||| regex anchor ||| code inserted after the first match``.
"""
import argparse
import os
import re
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
HERE = os.path.dirname(os.path.abspath(__file__))

STAMP_MACROS = r"""
#define TLS(stp, slot) do { if (threadIdx.x == 0) { unsigned long long _t; \
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(_t)); \
  atomicMin((unsigned long long *)((stp) + 32 + 2 * (slot)), _t); \
  atomicMax((unsigned long long *)((stp) + 33 + 2 * (slot)), _t); } } while (0)
#define TL(slot) TLS(st.state, slot)
"""


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--stamps", default=os.path.join(HERE, "stamps_decode.txt"))
    a = ap.parse_args()
    dst = os.path.abspath(a.out)
    shutil.rmtree(dst, ignore_errors=True)
    shutil.copytree(os.path.join(ROOT, "kiv_b200"), os.path.join(dst, "kiv_b200"),
                    ignore=shutil.ignore_patterns("*.so", "__pycache__", "timeline"))
    shutil.copytree(os.path.join(ROOT, "include"), os.path.join(dst, "include"))
    hdr = os.path.join(dst, "include/kiv_b200.h")
    s = open(hdr).read().replace("#define KIV_STATE_WORDS 32", "#define KIV_STATE_WORDS 160")
    open(hdr, "w").write(s)
    nat = os.path.join(dst, "kiv_b200/_native.py")
    s = open(nat).read().replace("STATE_WORDS = 32", "STATE_WORDS = 160")
    open(nat, "w").write(s)
    cm = os.path.join(dst, "kiv_b200/csrc/common.cuh")
    open(cm, "a").write(STAMP_MACROS)
    lines = [l for l in open(a.stamps).read().splitlines() if l.strip() and not l.startswith("#")]
    for line in lines:
        f, anchor, text = (x.strip() for x in line.split("|||"))
        p = os.path.join(dst, "kiv_b200/csrc", f)
        s = open(p).read()
        m = re.search(anchor, s, re.S)
        if not m:
            sys.exit(f"anchor not found in {f}: {anchor}")
        s = s[:m.end()] + "\n" + text + "\n" + s[m.end():]
        open(p, "w").write(s)
    r = subprocess.run(["make", "-C", os.path.join(dst, "kiv_b200/csrc"), "-j8", "BUILD=" + os.path.join(dst, "_build")],
                       capture_output=True, text=True)
    if r.returncode:
        sys.exit(r.stdout[-2000:] + r.stderr[-3000:])
    print("built", dst)


if __name__ == "__main__":
    main()
