"""CPU: safety properties of the CUDA sources that no GPU run should be
needed to establish.

* No bulk or tensor copy uses cluster multicast: the library runs on 2-8
  GPUs, and a multicast load whose source can be another GPU's memory is not
  allowed anywhere in it (commit multicast, `tcgen05.commit ... multicast`,
  is a different instruction and stays allowed).
* Every mbarrier poll goes through the bounded wait of h3b_common.cuh
  (`mbar_wait`, which gives up after a time budget, records the site in the
  status word and raises the abort flag): the raw try_wait helpers are called
  nowhere else, and the only unbounded-looking loop is that wait's own.
* No device-side trap or assert: failures are reported through the status
  word, never by killing the context.
* Every setmaxnreg split is checked against the launch's register budget by
  a static_assert in the same file.
"""
from __future__ import annotations

import re
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "minixmax_h3_b200" / "csrc"
SOURCES = sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cuh")])


def _code(path: Path) -> str:
    """The file without // and /* */ comments."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def test_sources_found():
    names = {p.name for p in SOURCES}
    assert {"gemm.cu", "attention.cu", "quant.cu", "elementwise.cu", "h3b_common.cuh"} <= names


def test_no_multicast_bulk_copies():
    for p in SOURCES:
        for n, line in enumerate(_code(p).splitlines(), 1):
            if "cp.async.bulk" in line:
                assert "multicast" not in line, f"{p.name}:{n}: {line.strip()}"


def test_mbarrier_polls_are_bounded():
    raw = re.compile(r"\bmbar_try_wait(_spin|_cluster)?\s*\(")
    for p in SOURCES:
        code = _code(p)
        calls = [m.start() for m in raw.finditer(code)]
        if p.name == "h3b_common.cuh":
            # the three definitions and their uses inside mbar_wait's poll lambda
            start = code.index("H3B_DEV bool mbar_wait(")
            end = code.index("\n}\n", start)
            for pos in calls:
                line = code[: pos].rsplit("\n", 1)[-1]
                assert line.startswith("H3B_DEV bool") or start < pos < end, f"{p.name}: raw poll outside mbar_wait"
        else:
            assert not calls, f"{p.name}: raw mbarrier poll outside the bounded wait"
        assert "try_wait" not in code.replace("mbar_try_wait", "") or p.name == "h3b_common.cuh", p.name


def test_only_the_bounded_wait_loops_forever():
    for p in SOURCES:
        code = _code(p)
        loops = len(re.findall(r"while\s*\(\s*(true|1)\s*\)|for\s*\(\s*;\s*;\s*\)", code))
        assert loops == (1 if p.name == "h3b_common.cuh" else 0), p.name
    common = _code(CSRC / "h3b_common.cuh")
    body = common[common.index("H3B_DEV bool mbar_wait("):]
    body = body[: body.index("\n}\n")]
    assert "H3B_WAIT_NS" in body and "abort_flag" in body and "return false" in body


def test_no_device_trap_or_assert():
    for p in SOURCES:
        code = _code(p)
        assert "__trap" not in code, p.name
        assert not re.search(r"(?<!static_)\bassert\s*\(", code), p.name
        assert "brkpt" not in code, p.name


def test_register_splits_are_statically_checked():
    for p in SOURCES:
        code = _code(p)
        if "setmaxnreg" in code:
            assert re.search(r"static_assert\([^;]*REGS_[A-Z]+[^;]*register split exceeds launch", code, re.S), p.name
