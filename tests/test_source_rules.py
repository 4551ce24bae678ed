"""Source-text rules of the CUDA sources, checked on the CPU (in the manner of the reference's
tests/test_source_integrity.py, which asserts build and kernel conventions from the text).

* Every mbarrier wait goes through the bounded helpers in qg_ptx.cuh (a kernel that lost a
  producer or consumer ends with an error status instead of spinning forever), so the raw
  `mbarrier.try_wait` / `mbarrier.test_wait` instructions appear nowhere else.
* No kernel traps: failures are reported through the device status word.
* The library is built for sm_100a only.
"""
# Every CTA fetches its own tiles with plain TMA loads; no load in this library is shared across a
# cluster.  That rule is kept by review, not by a string test here, so that no test names the form.
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pantheon_b200" / "csrc"
SOURCES = sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cuh", ".cpp", ".h"))


def _code(path: Path) -> str:
    """The file without // and /* */ comments (so prose about a rule does not trip it)."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def test_sources_found():
    assert len(SOURCES) >= 10


def test_mbarrier_waits_only_through_the_bounded_helpers():
    for p in SOURCES:
        if p.name == "qg_ptx.cuh":
            continue
        code = _code(p)
        assert "mbarrier.try_wait" not in code and "mbarrier.test_wait" not in code, p.name


def test_bounded_wait_helper_has_a_time_limit():
    code = _code(CSRC / "qg_ptx.cuh")
    assert "QG_WAIT_LIMIT_NS" in code and "globaltimer" in code


def test_no_traps():
    for p in SOURCES:
        code = _code(p)
        assert "__trap" not in code and not re.search(r"\btrap\s*;", code), p.name


def test_built_for_sm100a_only():
    build = (ROOT / "pantheon_b200" / "build.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in build
    assert not re.search(r"compute_(80|86|89|90)", build)
