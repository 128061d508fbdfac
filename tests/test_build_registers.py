"""ptxas register report of the GEMM kernels (no GPU needed: nvcc cross-compiles for sm_100a).

The bias / GELU / fp32 / peer-store epilogues keep the next chunk's tcgen05.ld in flight while the
current chunk is processed; its destination registers are written asynchronously until the
matching tcgen05.wait::ld, so none of them may ever be spilled. The test compiles the library with
-Xptxas -v and requires zero spill bytes for every kernel instantiation that uses that pattern.
"""

import re
import subprocess

from tiktoktechjam2026track3_b200.build import ARCH_FLAGS, CSRC_DIR, nvcc_path

DOUBLE_BUFFERED_EPILOGUES = {0, 1, 4, 5, 6, 7}


def test_double_buffered_gemm_epilogues_do_not_spill(tmp_path):
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-std=c++17", "-Xptxas=-v", "-Xcompiler", "-fPIC", "-shared",
           "-o", str(tmp_path / "probe.so"), str(CSRC_DIR / "b200tx.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-2000:]
    current = None
    checked = 0
    for line in proc.stderr.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            current = m.group(1)
            continue
        if current is None or "spill" not in line:
            continue
        k = re.match(r"_ZN2b21[45]gemm_tc2?_kernelILi(\d+)ELi(\d+)E", current)
        if k and int(k.group(2)) in DOUBLE_BUFFERED_EPILOGUES:
            checked += 1
            stores, loads = map(int, re.findall(r"(\d+) bytes spill (?:stores|loads)", line))
            assert stores == 0 and loads == 0, (current, line)
    assert checked >= 12


def test_attention_kernels_do_not_spill(tmp_path):
    """The tensor-core attention kernels hold a row's scores (and their packed exponentials) in
    registers across a tile; a spill there costs local-memory traffic on every score tile."""
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-std=c++17", "-Xptxas=-v", "-Xcompiler", "-fPIC", "-shared",
           "-o", str(tmp_path / "probe.so"), str(CSRC_DIR / "b200tx.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-2000:]
    current = None
    seen = set()
    for line in proc.stderr.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            current = m.group(1)
            continue
        if current is None or "spill" not in line:
            continue
        k = re.search(r"attention_(solo|wide)_kernel", current)
        if k:
            seen.add(k.group(1))
            stores, loads = map(int, re.findall(r"(\d+) bytes spill (?:stores|loads)", line))
            assert stores == 0 and loads == 0, (current, line)
    assert seen == {"solo", "wide"}
