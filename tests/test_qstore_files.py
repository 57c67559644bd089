"""On-disk QStore: the native positional reader, the layout validator against the
reference's verdicts, and the read oracle against the reference's outputs (no GPU)."""
from __future__ import annotations

import json
import shutil
from pathlib import Path

import numpy as np
import pytest

from oracle.qstore_files import StoreOracle

GOLDEN = Path(__file__).resolve().parent / "golden"
STORE = GOLDEN / "qstore_small"


# The reference validator's error text (its verdict on each corrupted store, recorded in the
# fixture) mapped to the rule it enforces and the block or file it names. The B200 validator
# raises QStoreLayoutError with its own wording; what must agree is accept/reject, the broken
# rule and where it was found.
_REFERENCE_RULES = [
    (r"must declare dtype", "header", None),
    (r"requires config and a non-empty block table", "header", None),
    (r"requires qrow and fp32 blocks", "kinds", None),
    (r"block field '\w+' must be", "field", "*"),
    (r"block shape", "shape", "*"),
    (r"qrow '(.+)' (weight length|scale range) does not match", "length", 1),
    (r"fp32 '(.+)' range does not match", "length", 1),
    (r"block '(.+)' has unsupported kind", "kind", 1),
    (r"alias '(.+)' targets missing block", "alias-target", 1),
    (r"alias cycle contains '(.+)'", "alias-cycle", "cycle"),
    (r"file is missing: (\S+)", "missing-file", 1),
    (r"(\S+) range for block '(.+)' exceeds file bounds", "bounds", 2),
    (r"(\S+) ranges overlap at block '(.+)'", "overlap", 2),
    (r"(\S+) has an unreferenced gap before block '(.+)'", "gap", 2),
    (r"(\S+) block ranges do not cover the complete file", "tail", 1),
]


def _expected(verdict: str, case: dict):
    import re

    for pattern, reason, subject in _REFERENCE_RULES:
        m = re.search(pattern, verdict)
        if not m:
            continue
        if isinstance(subject, int):
            return reason, m.group(subject)
        if subject == "cycle":  # any member of the cycle the case builds
            return reason, {edit[1] for edit in case["edit"] if edit[0] == "alias"}
        if subject == "*":  # the block the case edited
            return reason, {edit[1] for edit in case["edit"] if edit[0] == "set"}
        return reason, None
    raise AssertionError(f"no rule recognised in reference verdict {verdict!r}")


def test_layout_validator_matches_reference_verdicts(tmp_path):
    import sys

    sys.path.insert(0, str(GOLDEN))
    from make_qstore_fixtures import apply_case

    from mrun_b200.qstore import LAYOUT_REASONS, QStoreLayoutError, validate_int8_layout

    cases = json.loads((GOLDEN / "qstore_layout_cases.json").read_text())
    assert len(cases) >= 10 and cases[0]["verdict"] == "ok"
    seen = set()
    for i, case in enumerate(cases):
        directory = tmp_path / f"case{i}"
        apply_case(STORE, directory, case)
        manifest = json.loads((directory / "manifest.json").read_text())
        if case["verdict"] == "ok":
            validate_int8_layout(directory, manifest)
            continue
        assert case["verdict"].startswith("RuntimeError: ")
        with pytest.raises(RuntimeError) as err:
            validate_int8_layout(directory, manifest)
        assert isinstance(err.value, QStoreLayoutError), case["name"]
        reason, subject = _expected(case["verdict"], case)
        assert err.value.reason == reason, (case["name"], str(err.value))
        assert err.value.reason in LAYOUT_REASONS
        if isinstance(subject, set):
            assert err.value.subject in subject, (case["name"], str(err.value))
        elif subject is not None:
            assert err.value.subject == subject, (case["name"], str(err.value))
        seen.add(reason)
    assert len(seen) >= 10  # the fixture exercises most rules


def test_oracle_pinned_to_reference_outputs(golden):
    g = golden("qstore")
    oracle = StoreOracle(STORE)
    for name, block in oracle.blocks.items():
        key = name.replace(".", "_")
        if block.get("kind") == "fp32":
            np.testing.assert_array_equal(oracle.fp32(name), g["fp32__" + key])
        else:
            np.testing.assert_array_equal(oracle.weight(name), g["weight__" + key])
    np.testing.assert_array_equal(oracle.embed_rows("model.embed_tokens.weight", g["embed_ids"]), g["embed_rows"])


def test_native_reader_bit_exact(tmp_path):
    from mrun_b200.qstore import StoreFile

    rng = np.random.default_rng(5)
    data = rng.integers(0, 256, (37 << 20) + 4099, dtype=np.uint8)  # > 8 pieces of 4 MiB, ragged end
    path = tmp_path / "blob.bin"
    data.tofile(path)
    f = StoreFile(path)
    assert f.size == data.size
    for offset, nbytes, threads in [(0, data.size, 1), (0, data.size, 8), (12345, 20 << 20, 3), (data.size - 7, 7, 4),
                                    (1, 1, 16), (8 << 20, 0, 2), (3, (9 << 20) + 1, 64)]:
        dst = np.zeros(max(nbytes, 1), dtype=np.uint8)
        f.read_into(offset, nbytes, dst, threads=threads, drop_after=(threads % 2 == 0))
        np.testing.assert_array_equal(dst[:nbytes], data[offset:offset + nbytes])
    with pytest.raises(ValueError, match="beyond"):
        f.read_into(data.size - 3, 4, np.zeros(4, np.uint8))
    with pytest.raises(ValueError, match="destination holds"):
        f.read_into(0, 8, np.zeros(4, np.uint8))
    f.advise(0, 1 << 20, will_need=True)
    f.advise(0, 1 << 20, will_need=False)
    f.close()
    f.close()  # idempotent
    with pytest.raises(ValueError, match="closed"):
        f.read_into(0, 1, np.zeros(1, np.uint8))
    with pytest.raises(OSError, match="No such file"):
        StoreFile(tmp_path / "missing.bin")
    with pytest.raises(ValueError, match="regular file"):
        StoreFile(tmp_path)


def test_native_reader_concurrent_callers(tmp_path):
    """Several threads read one handle at once (pread keeps no shared offset)."""
    from concurrent.futures import ThreadPoolExecutor

    from mrun_b200.qstore import StoreFile

    data = np.random.default_rng(6).integers(0, 256, 24 << 20, dtype=np.uint8)
    path = tmp_path / "blob.bin"
    data.tofile(path)
    f = StoreFile(path)
    spans = [(i * (3 << 20) + 11, (2 << 20) + 5) for i in range(7)]

    def read(span):
        out = np.empty(span[1], np.uint8)
        f.read_into(span[0], span[1], out, threads=4)
        return out

    with ThreadPoolExecutor(4) as pool:
        for (off, n), got in zip(spans, pool.map(read, spans)):
            np.testing.assert_array_equal(got, data[off:off + n])
    f.close()


def test_writer_round_trip(tmp_path):
    """write_qstore lays blocks back to back; the validator accepts it and the oracle reads
    back exactly the arrays written."""
    from mrun_b200.qstore import load_manifest
    from mrun_b200.qstore_build import write_qstore

    rng = np.random.default_rng(9)
    codes = rng.integers(-127, 128, (33, 48), dtype=np.int8)
    scales = rng.random(33).astype(np.float32)
    norm = rng.random(48).astype(np.float32)
    write_qstore(tmp_path / "m", qrows={"a": (codes, scales), "b": (codes[:5], scales[:5])}, fp32={"n": norm},
                 aliases={"c": "a"}, config={"hidden_size": 48})
    man = load_manifest(tmp_path / "m")
    assert man["blocks"]["b"]["w_off"] == codes.nbytes
    oracle = StoreOracle(tmp_path / "m")
    np.testing.assert_array_equal(oracle.qrow("c")[0], codes)
    np.testing.assert_array_equal(oracle.qrow("b")[1], scales[:5])
    np.testing.assert_array_equal(oracle.fp32("n"), norm)
    shutil.rmtree(tmp_path / "m")


def test_ring_slot_freed_after_staging_error():
    """A failed staging read reaches the caller of take() and frees its slot."""
    from concurrent.futures import Future

    from mrun_b200.qstore import _RingSlot

    class _Ring:  # the take() path of the ring without a device: a slot whose staging failed
        from mrun_b200.qstore import _PageRing as _cls
        take = _cls.take

    ring = _Ring()
    slot = _RingSlot()
    slot.name, slot.shape = "w", (2, 2)
    fut = Future()
    fut.set_exception(OSError("store_file_read: Input/output error"))
    slot.future = fut
    ring.inflight = {"w": slot}
    ring.stats = {"hits": 0, "late_hits": 0, "misses": 0}
    with pytest.raises(OSError, match="Input/output"):
        ring.take("w")
    assert slot.name is None and slot.future is None and ring.stats["hits"] == 1


def test_resident_page_cache_policies():
    """pin-fill admits while the budget allows and never evicts; lru evicts the oldest page."""
    from mrun_b200.qstore import ResidentPageCache

    pin = ResidentPageCache(250, "pin-fill")
    for i in range(4):
        pin.put(f"b{i}", f"page{i}", 100)
    assert list(pin.pages) == ["b0", "b1"] and pin.stats["rejected"] == 2 and pin.get("b3") is None
    assert pin.get("b0") == "page0" and pin.stats["hits"] == 1
    lru = ResidentPageCache(250, "lru")
    for i in range(3):
        lru.put(f"b{i}", f"page{i}", 100)
    assert list(lru.pages) == ["b1", "b2"] and lru.stats["evicted"] == 1
    lru.get("b1")
    lru.put("b3", "page3", 100)
    assert list(lru.pages) == ["b1", "b3"] and lru.bytes == 200
    lru.put("huge", "x", 1000)
    assert "huge" not in lru.pages and lru.stats["rejected"] == 1
    with pytest.raises(ValueError, match="unknown cache policy"):
        ResidentPageCache(10, "mru")
