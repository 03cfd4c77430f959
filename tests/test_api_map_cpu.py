"""The reference-to-framework import map printed in the README resolves: every reference symbol has its
counterpart at the listed module here (and, with the reference installed, exists at the listed
reference module), so a user of the reference can switch by changing imports."""
import importlib
import re
from pathlib import Path

import pytest

from _oracle import needs_reference, ref

README = Path(__file__).resolve().parents[1] / "README.md"
ROW = re.compile(r"^\| `([\w.]+)` \| `([\w.]+)` \| (.+) \|$")


def _rows():
    rows = []
    for line in README.read_text().splitlines():
        m = ROW.match(line.strip())
        if m:
            names = [n.strip(" `") for n in m.group(3).split(",")]
            rows.append((m.group(1), m.group(2), names))
    return rows


ROWS = _rows()


def test_the_readme_has_an_import_map():
    assert len(ROWS) >= 20


@pytest.mark.parametrize("ref_module,our_module,names", ROWS, ids=[r[0] for r in ROWS])
def test_every_listed_symbol_exists_here(ref_module, our_module, names):
    mod = importlib.import_module(our_module)
    for name in names:
        assert hasattr(mod, name), f"{our_module}.{name}"


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("ref_module,our_module,names", ROWS, ids=[r[0] for r in ROWS])
def test_every_listed_symbol_exists_in_the_reference(ref_module, our_module, names):
    ref()
    mod = importlib.import_module(ref_module)
    for name in names:
        assert hasattr(mod, name), f"{ref_module}.{name}"
