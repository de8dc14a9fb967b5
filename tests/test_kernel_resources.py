"""Resource assumptions of the sm_100a kernels, read from ptxas's report at
build time (no GPU needed).

* The attention kernel moves registers between its warpgroups with
  `setmaxnreg`; the split is only satisfiable when every thread launches with
  the register count the kernel's constants name (the host refuses to launch
  it otherwise, so a change that moves the count would only show on a GPU).
* The hot kernels keep their working set in registers: no local-memory
  spills in the attention, GEMM, split-K, int8-weight GEMM and GEMV kernels.
"""
from __future__ import annotations

import concurrent.futures as cf
import re
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

import __graft_entry__ as ge

CSRC = Path(ge.__file__).resolve().parent / "iree-hexagon-plugins_b200" / "csrc"


def _ptxas_report(src: Path) -> dict[str, tuple[int, int, int]]:
    """{mangled kernel name: (registers, spill-store bytes, spill-load bytes)}."""
    build = ge._load_build_module()
    try:
        nvcc = build._nvcc()
    except RuntimeError:
        pytest.skip("nvcc not available")
    with tempfile.TemporaryDirectory() as tmp:
        r = subprocess.run([nvcc, *build.NVCC_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o",
                            str(Path(tmp) / "k.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    report: dict[str, tuple[int, int, int]] = {}
    name = None
    spills = (0, 0)
    for line in r.stderr.splitlines():
        m = re.search(r"Function properties for (\S+)", line)
        if m:
            name, spills = m.group(1), (0, 0)
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and name:
            spills = (int(m.group(1)), int(m.group(2)))
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and name:
            report[name] = (int(m.group(1)), *spills)
            name = None
    return report


@pytest.fixture(scope="module")
def reports():
    if shutil.which("nvcc") is None and not Path("/usr/local/cuda/bin/nvcc").exists():
        pytest.skip("nvcc not available")
    srcs = [CSRC / "attention.cu", CSRC / "gemm.cu"]
    with cf.ThreadPoolExecutor(len(srcs)) as ex:
        return dict(zip((s.name for s in srcs), ex.map(_ptxas_report, srcs)))


def _kernels(report, fragment):
    found = {k: v for k, v in report.items() if fragment in k}
    assert found, f"no kernel matching {fragment!r} in the ptxas report"
    return found


def test_attention_launch_registers_match_the_register_split(reports):
    text = (CSRC / "attention.cu").read_text()
    launch = int(re.search(r"constexpr int kAttRegsLaunch = (\d+);", text).group(1))
    for name, (regs, st, ld) in _kernels(reports["attention.cu"], "attention_fwd_kernel").items():
        assert regs == launch, f"{name}: {regs} registers at launch, the split assumes {launch}"


@pytest.mark.parametrize("src,fragment", [
    ("attention.cu", "attention_fwd_kernel"),
    ("attention.cu", "attention_decode_kernel"),
    ("gemm.cu", "gemm_sm100_kernel"),
    ("gemm.cu", "gemm_splitk_sm100_kernel"),
    ("gemm.cu", "gemm_w8_sm100_kernel"),
    ("gemm.cu", "gemv_w8_sk_kernel"),
])
def test_hot_kernels_do_not_spill(reports, src, fragment):
    for name, (regs, st, ld) in _kernels(reports[src], fragment).items():
        assert st == 0 and ld == 0, f"{name}: {st} B spill stores, {ld} B spill loads"
