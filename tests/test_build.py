"""Reproducible build (the reference requires its cubin to build to identical bytes twice): the library
built twice from the same sources, into two separate directories, is byte-identical."""
import hashlib


def _sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def test_library_builds_to_identical_bytes(tmp_path):
    from macuda_b200 import build as b
    one = b.build(force=True, lib_path=str(tmp_path / "a" / "libtinycublas_b200.so"), build_dir=str(tmp_path / "a"))
    two = b.build(force=True, lib_path=str(tmp_path / "b" / "libtinycublas_b200.so"), build_dir=str(tmp_path / "bb"))
    assert _sha(one) == _sha(two)
