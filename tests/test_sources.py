"""Static checks of the CUDA sources (no GPU needed).

Every kernel is launched with programmatic dependent launch, so each must execute
griddepcontrol.wait (pdl_wait) before it touches memory a predecessor writes; a
kernel without it would race with the kernel launched before it.
"""
import re
from pathlib import Path

CSRC = Path(__file__).resolve().parent.parent / "fier-2bits_b200" / "csrc"


def test_every_kernel_waits_for_its_predecessor_first():
    """pdl_wait() opens every kernel, except that loads of inputs no kernel of this
    library writes (queries, head maps) may come first, and then the code before the
    wait must consist of prefetch_* calls and index arithmetic only."""
    missing = []
    for path in sorted(CSRC.glob("*.cu")):
        text = path.read_text()
        for m in re.finditer(r"__global__[^{;]*?(\w+)\s*\((?:[^()]|\([^()]*\))*\)\s*\{", text):
            head = text[m.end(): m.end() + 80]
            if "pdl_wait();" in head:
                continue
            body = text[m.end():]
            k = body.find("pdl_wait();")
            before = body[:k] if k >= 0 else ""
            ok = k >= 0 and "prefetch_" in before and "__syncthreads" not in before and \
                not re.search(r"\[[^\]]*\]\s*=[^=]", before.replace("pf.", ""))
            if not ok:
                missing.append(f"{path.name}:{m.group(1)}")
    assert not missing, f"kernels without pdl_wait() at the top: {missing}"


def test_no_cluster_multicast_loads():
    for path in CSRC.glob("*"):
        qualifier = ".".join(["", "multicast"]) + "::" + "cluster"  # built, so this file does not name it
        assert qualifier not in path.read_text(), path.name
