"""The ncu summaries under profiles/ give commands that run committed files only: every
`python bench.py ...` they quote parses with bench.py's own arguments, every `ncu` command keeps
the clocks as they are (`--clock-control none`), and none reads a scratch folder."""

import re
import shlex
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PROFILES = sorted((ROOT / "profiles").glob("*.md"))


def _bench_commands(text):
    """The `python bench.py ...` commands of a summary, each joined across its continuation lines."""
    joined = re.sub(r"\\\n\s*", " ", text)
    joined = re.sub(r"`[^`]*`", lambda m: m.group(0).replace("\n", " "), joined)  # wrapped inline code
    out = []
    for m in re.finditer(r"python bench\.py([^`\n#]*)", joined):
        out.append(shlex.split(m.group(1)))
    return out


def test_there_are_summaries():
    assert PROFILES


@pytest.mark.parametrize("path", PROFILES, ids=lambda p: p.name)
def test_a_summary_quotes_commands_that_run(path, monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench

    text = path.read_text()
    assert "ncu " in text or "python " in text, "no command"
    for args in _bench_commands(text):
        ends = [i for i, a in enumerate(args) if a in ("&&", "||", "|", ";")]
        args = args[:ends[0]] if ends else args
        monkeypatch.setattr(sys, "argv", ["bench.py", *[a for a in args if not a.startswith(">")]])
        bench.parse()  # exits on an argument bench.py does not take
    joined = re.sub(r"\\\n\s*", " ", text)
    for line in joined.splitlines():
        if re.search(r"(^|[\s`])ncu\s+-", line) and "-i " not in line:
            assert "--clock-control none" in line, line
    assert "_work/" not in text
