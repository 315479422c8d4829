"""Runs the C++ contract suite (StorageRuntime vs the mock DataPath kit, object store, config spec)."""
import os
import subprocess

import pytest

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tutti_b200", "bin",
                   "tutti_native_tests")


def test_native_contract_suite():
    if not os.path.exists(BIN):
        from tutti_b200 import build_native

        build_native.build(["tutti_native_tests"])
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout
