"""CPU: structural rules of the kernel sources that a fault would otherwise
have to reveal.

elect.sync (`elect_one()`) names all 32 lanes (member mask 0xffffffff), so it
must be executed by a converged warp: never inside a block entered by one lane
(`if (lane == 0)`, `if (threadIdx.x == 0)` ...). Executed from a single lane it
is undefined behaviour, the most probable cause of the "illegal instruction"
an early-load prologue variant raised (its TMA issue, guarded by elect_one(),
sat inside the lane-0 barrier-initialisation block).
"""
import re
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "tilemix-cuda_b200" / "csrc"
LANE_GUARD = re.compile(r"if\s*\(([^{;]*)\)\s*\{?\s*$")
SINGLE_LANE = re.compile(r"\blane\s*==|\bthreadIdx\.x\s*==|\blane_id\(\)\s*==")


def enclosing_conditions(text: str, pos: int) -> list[str]:
    """Conditions of the `if` blocks (braced or not) enclosing text[pos]."""
    conds, depth = [], 0
    i = pos
    # braced blocks: walk back, tracking brace depth
    while i > 0:
        i -= 1
        c = text[i]
        if c == "}":
            depth += 1
        elif c == "{":
            if depth == 0:
                line_start = text.rfind("\n", 0, i) + 1
                header = text[line_start:i + 1]
                m = re.search(r"if\s*\((.*)\)\s*\{$", header.strip())
                if m:
                    conds.append(m.group(1))
            else:
                depth -= 1
    # an unbraced `if (...)` on the same line as the call
    line_start = text.rfind("\n", 0, pos) + 1
    m = re.search(r"if\s*\((.*)\)\s*$", text[line_start:pos])
    if m:
        conds.append(m.group(1))
    return conds


def test_elect_sync_is_never_issued_from_a_single_lane():
    checked = 0
    for path in sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")):
        text = path.read_text()
        for m in re.finditer(r"elect_one\(\)", text):
            if text[max(0, m.start() - 40):m.start()].rstrip().endswith("bool"):
                continue          # the definition
            bad = [c for c in enclosing_conditions(text, m.start()) if SINGLE_LANE.search(c)]
            assert not bad, f"{path.name}: elect_one() under a single-lane condition {bad}"
            checked += 1
    assert checked >= 5
