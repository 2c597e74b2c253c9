"""Process isolation (mirrors the reference's tests/test_isolation.py)."""

from __future__ import annotations

import sys

from avo.isolation import RESULT_PREFIX, extract_payload, run_json_worker


def test_worker_success_payload():
    code = f"print('noise'); print('{RESULT_PREFIX}' + '{{\"x\": 1}}')"
    result = run_json_worker([sys.executable, "-c", code], timeout_s=30)
    assert result.ok and result.payload == {"x": 1}


def test_worker_timeout_is_contained():
    result = run_json_worker([sys.executable, "-c", "import time; time.sleep(5)"], timeout_s=1)
    assert result.timed_out and not result.ok and result.returncode is None


def test_worker_crash_is_contained():
    result = run_json_worker([sys.executable, "-c", "import os; os._exit(139)"], timeout_s=30)
    assert result.returncode == 139 and not result.ok and result.payload is None


def test_payload_extraction_takes_last_line_and_rejects_garbage():
    text = f"{RESULT_PREFIX}{{\"a\": 1}}\n{RESULT_PREFIX}{{\"a\": 2}}\n"
    assert extract_payload(text) == {"a": 2}
    assert extract_payload(f"{RESULT_PREFIX}not json") is None
    assert extract_payload(f"{RESULT_PREFIX}[1, 2]") is None
    assert extract_payload("nothing here") is None
