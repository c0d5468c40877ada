"""Per-shape kernel selection cache (c3_b200.tuning): key format, JSON round trip, versioning
and installation into the library's table (no GPU needed for any of these)."""
import json

from c3_b200 import _lib, tuning


def test_key_is_sha256_of_a_versioned_description():
    k = tuning.gemm_key(16384, 4096, 4096, 0, 0, 0)
    assert len(k) == 64 and all(c in "0123456789abcdef" for c in k)
    assert k == tuning.gemm_key(16384, 4096, 4096, 0, 0, 0)
    assert k != tuning.gemm_key(16384, 4096, 4096, 0, 1, 0)


def test_json_round_trip_and_merge(tmp_path):
    p = tmp_path / "tune.json"
    e1 = {tuning.gemm_key(256, 512, 256, 0, 0, 1): {"M": 256, "N": 512, "K": 256, "a_mn": 0, "b_mn": 0,
                                                   "epilogue": 1, "variant": 2, "us": {"0": 5.0}}}
    e2 = {tuning.gemm_key(128, 256, 64, 1, 1, 2): {"M": 128, "N": 256, "K": 64, "a_mn": 1, "b_mn": 1,
                                                  "epilogue": 2, "variant": 1, "us": {"1": 3.0}}}
    tuning.write(e1, p)
    tuning.write(e2, p)
    data = tuning.read(p)
    assert data["version"] == tuning.VERSION
    assert set(data["entries"]) == set(e1) | set(e2)
    assert tuning.load(p) == 2
    _lib.load().c3cu_gemm_tune_clear()


def test_other_versions_are_ignored(tmp_path):
    p = tmp_path / "old.json"
    p.write_text(json.dumps({"version": "c3_tune_v0", "entries": {"x": {}}}))
    assert tuning.read(p) == {}
    assert tuning.load(p) == 0
    p.write_text("not json")
    assert tuning.read(p) == {}


def test_tune_set_rejects_unknown_variants():
    L = _lib.load()
    assert L.c3cu_gemm_tune_set(1, 1, 1, 0, 0, 0, 3) != 0
    assert L.c3cu_gemm_tune_set(1, 1, 1, 0, 0, 0, 2) == 0
    assert L.c3cu_gemm_tune_clear() == 0
