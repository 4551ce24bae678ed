"""Read the recorded binary runs with the reference runner itself; write what it decided.

    python tests/golden/make_runner_readings.py

Input: tests/golden/binary_runs.json (real stdout / stderr / exit codes of the
drop-in binaries on a B200, from capture_binary_runs.py).  For each run this
records, from the reference runner module (pantheon.py, found as
tests/reference_runner.py describes):
  * parse_kernel_output(stdout, stderr, returncode, test)  (pantheon.py:3421-3513)
    -> score, unit, status, error flag, the lines it keeps for the log;
  * the GPU verdict of a result row built from it with build_result_row
    (pantheon.py:3552) and judged by assess_gpu (pantheon.py:1303-1460), once
    with the runner as shipped and once after pantheon_b200.runner_hook.install.
Output: tests/golden/runner_readings.json, which the CPU tests compare with the
restated reader the GPU tests use (tests/contract_parse.py), so that reader is
pinned to the runner's own decisions on real outputs.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def readings(runner, runs):
    """The runner's reading of each run; `runner` is left as it was given."""
    from pantheon_b200 import runner_hook
    out = []
    for run in runs:
        score, unit, status, had_error, lines = runner.parse_kernel_output(run["stdout"], run["stderr"],
                                                                           run["returncode"], run["test"])
        row = runner.build_result_row(run["test"], 0, 2, 50, score, unit, {}, status=status)
        shipped = runner.assess_gpu([row], 0, "NVIDIA B200")["verdict"]
        added = runner_hook.install(runner)
        row.update(runner_hook.row_fields(run["test"], run["stdout"]))
        hooked = runner.assess_gpu([row], 0, "NVIDIA B200")["verdict"]
        runner.DIAGNOSTIC_TESTS.difference_update(added)
        out.append({"case": run["case"], "score": score, "unit": unit, "status": status, "had_error": had_error,
                    "kept_lines": lines, "verdict_shipped": shipped, "verdict_with_hook": hooked,
                    "sdc_mismatches": row.get(runner_hook.ROW_FIELD)})
    return out


def main() -> int:
    from tests.reference_runner import load_runner
    runner = load_runner()
    if runner is None:
        print("no reference runner found (set PANTHEON_REFERENCE)", file=sys.stderr)
        return 1
    runs = json.loads((HERE / "binary_runs.json").read_text())
    (HERE / "runner_readings.json").write_text(json.dumps(readings(runner, runs), indent=1) + "\n")
    print(f"wrote {len(runs)} readings")
    return 0


if __name__ == "__main__":
    sys.exit(main())
