"""Every `file:line` citation of a reference file in the product, the tests
and the docs stays inside that file.  The table holds the line counts of the
reference's files (tri_sds at the surveyed revision), so the check runs
without the reference checkout."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REF_LINES = {
    "worker.py": 68, "__init__.py": 10, "model.py": 135, "norm.py": 72, "train_eagle.py": 182,
    "fused_block.py": 243, "fused_qwen_decode.py": 309, "attention.py": 318, "qwen_model.py": 209,
    "eagle_head.py": 129, "draft_step.py": 85, "pyproject.toml": 20, "README.md": 36,
}
# a bare name (no directory before it) is a reference file; this repository's
# own files are cited with their directory (tri_sds_b200/model.py)
CITE = re.compile(r"(?<![\w/])(?:tri_sds/(?:triton_kernels/)?)?([A-Za-z_]+\.(?:py|toml|md)):(\d+)(?:-(\d+))?"
                  r"((?:,\s*\d+(?:-\d+)?)*)")
SKIP_DIRS = {".git", "_work", "gpurun_out", "__pycache__", "_build", "baseline", ".pytest_cache"}
# records written by others (the survey, reviews, driver output) are not checked here
SKIP_FILES = {"SURVEY.md", "VERDICT.md", "ADVICE.md", "BASELINE.md"}


def _files():
    for dp, dn, fn in os.walk(ROOT):
        dn[:] = [d for d in dn if d not in SKIP_DIRS]
        for f in fn:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".md", ".toml")) and f not in SKIP_FILES:
                yield os.path.join(dp, f)


def test_reference_citations_are_in_range():
    bad = []
    for p in _files():
        with open(p, errors="ignore") as fh:
            for i, line in enumerate(fh, 1):
                for m in CITE.finditer(line):
                    name = m.group(1)
                    if name not in REF_LINES:
                        continue
                    nums = [int(m.group(2))] + ([int(m.group(3))] if m.group(3) else [])
                    nums += [int(x) for x in re.findall(r"\d+", m.group(4) or "")]
                    if max(nums) > REF_LINES[name]:
                        bad.append(f"{os.path.relpath(p, ROOT)}:{i}: {m.group(0)}")
    assert not bad, "citations past the end of the reference file:\n" + "\n".join(bad)
