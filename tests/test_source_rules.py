"""Guard on the shipped sources (CPU): the product path does not import the oracle.

Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU legs may use ``oracle/``; the
package under ``avo-ampere_b200`` must fail loudly without its CUDA library instead of
routing through a CPU restatement.
"""

from __future__ import annotations

from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_product_path_does_not_import_the_oracle():
    product = [p for p in (ROOT / "avo-ampere_b200").rglob("*.py")]
    hits = [str(p) for p in product if "attention_oracle" in p.read_text(errors="ignore")
            or "from oracle" in p.read_text(errors="ignore")]
    assert hits == []
