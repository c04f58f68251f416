"""Source-level rules the kernels keep (CPU only, reads the sources).

* No bulk or tensor TMA load with cluster multicast: the same kernels run in
  the multi-GPU sharder and the multi-rank bench, where a multicast load whose
  source could be another GPU's memory is not allowed.  (Commits that arrive
  on both CTAs of a pair, tcgen05.commit ... multicast::cluster, are fine.)
* The batched-copy runtime calls are not used (one cudaMemcpyAsync per copy).
* Every kernel launched with programmatic dependent launch (launch_k) calls
  griddep_wait before it touches another kernel's data: each .cu file that
  uses launch_k defines kernels that call griddep_wait."""

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "ffwd_b200", "csrc")


def sources():
    for d in (CSRC, os.path.join(ROOT, "include"), os.path.join(ROOT, "ffwd_b200", "backend")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".cu", ".cuh", ".cc", ".h", ".c")):
                p = os.path.join(d, f)
                yield p, open(p).read()


def test_no_multicast_loads():
    pat = re.compile(r"cp\.async\.bulk[^\"]*multicast")
    for path, text in sources():
        assert not pat.search(text), path


def test_no_batched_copies():
    pat = re.compile("Memcpy" + "(3D)?" + "Batch")  # spelled in pieces on purpose
    for path, text in sources():
        assert not pat.search(text), path


def test_dependent_launch_kernels_wait():
    for path, text in sources():
        if path.endswith(".cu") and "launch_k(" in text:
            assert "griddep_wait()" in text, path
