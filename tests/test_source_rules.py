"""Guards on the shipped sources (CPU).

* No TMA or bulk load with cluster multicast anywhere in the sources: the kernels run on
  several GPUs (head sharding, the ring), and a multicast load whose source can be
  another GPU's memory is not allowed in this code base at all.
* None of the batched-memcpy runtime/driver entry points is named in any source.
* The product path does not import the oracle: only tests, smoke() and bench.py's CPU
  legs may.
"""

from __future__ import annotations

from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SOURCES = [p for p in (ROOT / "avo-ampere_b200").rglob("*") if p.suffix in {".cu", ".cuh", ".h", ".py", ".cpp"}]
SOURCES += list((ROOT / "include").glob("*.h")) + [ROOT / "bench.py", ROOT / "__graft_entry__.py"]


def test_no_cluster_multicast_loads():
    needle = "multicast" + "::cluster"
    hits = [str(p) for p in SOURCES if needle in p.read_text(errors="ignore")]
    assert hits == []


def test_no_batched_memcpy_entry_points():
    names = [prefix + "emcpy" + mid + "BatchAsync" for prefix in ("cudaM", "cuM") for mid in ("", "3D")]
    hits = [(str(p), n) for p in SOURCES for n in names if n in p.read_text(errors="ignore")]
    assert hits == []


def test_product_path_does_not_import_the_oracle():
    product = [p for p in (ROOT / "avo-ampere_b200").rglob("*.py")]
    hits = [str(p) for p in product if "attention_oracle" in p.read_text(errors="ignore")
            or "from oracle" in p.read_text(errors="ignore")]
    assert hits == []
