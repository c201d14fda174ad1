"""Repository lint: no TMA or bulk-copy load that broadcasts to a thread-block cluster
anywhere in the sources.

Such a load whose source can be another GPU's memory (peer buffers, symmetric memory) has
hung GPUs. Keeping every bulk/TMA copy free of the cluster-broadcast qualifier rules it out by
construction, including for kernels that today only read local memory. A tcgen05 commit
with that qualifier is an mbarrier arrive, not a load, and stays allowed. (The instruction
tokens are assembled at run time so this file spells no such load itself.)
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXTS = (".cu", ".cuh", ".h", ".hpp", ".cpp", ".cc", ".py")
SKIP_DIRS = {".git", "_work", "build", "gpurun_out", "baseline", "__pycache__", ".pytest_cache"}
BULK = "cp.async" + ".bulk"
MCAST = "".join(["multi", "cast", ":", ":", "clus", "ter"])  # assembled: no literal qualifier here


def _sources():
    for d, subdirs, files in os.walk(ROOT):
        subdirs[:] = [s for s in subdirs if s not in SKIP_DIRS]
        for f in files:
            if f.endswith(EXTS):
                yield os.path.join(d, f)


def _statements(text):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = "\n".join(line.split("//")[0] if "//" in line and "://" not in line else line
                     for line in text.splitlines())
    # inline-PTX strings may split one instruction over several C string literals / lines
    joined = re.sub(r'"\s*\n\s*"', "", text)
    return joined.split(";")


def _offending(text):
    return [s.strip() for s in _statements(text) if BULK in s and MCAST in s]


def test_no_cluster_broadcast_copies():
    bad = []
    for path in _sources():
        with open(path, encoding="utf-8", errors="ignore") as fh:
            text = fh.read()
        if MCAST not in text:
            continue
        bad += [f"{os.path.relpath(path, ROOT)}: {s[:120]}" for s in _offending(text)]
    assert not bad, "cluster-broadcast bulk/TMA copies are not allowed:\n" + "\n".join(bad)


def test_lint_catches_a_broadcast_copy():
    load = ('asm volatile("' + BULK + '.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"\n'
            '             ".' + MCAST + ' [%0], [%1, {%2, %3}], [%4], %5;")')
    assert _offending(load)
    commit = 'asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.' + MCAST + '.b64 [%0];")'
    assert not _offending(commit)
    commented = "// " + BULK + " ... " + MCAST + " would be banned\nint x;"
    assert not _offending(commented)
