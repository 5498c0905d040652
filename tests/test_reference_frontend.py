"""Drop-in check on the CPU: the reference's own Python frontend
(python/cubutterfly/__init__.py and rns.py of the reference tree, imported
unchanged from there) binds libcubutterfly_b200.so, builds and validates
descriptors through it and reads back the same JSON this build's frontend
produces.  Skipped where the reference tree is absent (GPU hosts run the
prebuilt files only).  Also covers `python -m cubutterfly_b200`."""
import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import pytest

import cubutterfly_b200 as cb
from oracle.oracle import default_reference_root

REF_PY = Path(default_reference_root()) / "python" / "cubutterfly"


def load_reference_package():
    if not (REF_PY / "__init__.py").is_file():
        pytest.skip("reference tree not present on this host")
    spec = importlib.util.spec_from_file_location("ref_cubutterfly", REF_PY / "__init__.py",
                                                  submodule_search_locations=[str(REF_PY)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_cubutterfly"] = mod
    spec.loader.exec_module(mod)
    return mod


CASES = [
    dict(op=0, extents=[4096], batch=1024),
    dict(op=2, storage=1, compute=1, extents=[4096], batch=16384, output_scale=1 / 64, output_rounding=1),
    dict(op=3, storage=8, extents=[1 << 24], batch=16, in_place=True),
    dict(op=1, storage=9, extents=[1 << 16], batch=32, modulus=576460756061519873, output_orders=[1]),
    dict(op=0, extents=[1 << 30], batch=1, inverse=True),
]


@pytest.mark.parametrize("fields", CASES)
def test_reference_frontend_binds_this_library(lib, fields):
    ref = load_reference_package()
    rlib = ref.Library(str(cb.DEFAULT_LIBRARY))
    with ref.Descriptor(rlib, ref.Transform(**fields)) as d:
        d.validate()
        theirs = json.loads(d.json())
        caps = json.loads(d.capabilities_json())
    with cb.Descriptor(lib, cb.Transform(**fields)) as d:
        ours = json.loads(d.json())
    assert theirs == ours
    assert caps


def test_reference_frontend_sees_our_errors(lib):
    ref = load_reference_package()
    rlib = ref.Library(str(cb.DEFAULT_LIBRARY))
    with ref.Descriptor(rlib, ref.Transform(op=0, extents=[0], batch=1)) as d:
        with pytest.raises(ref.Error) as e:
            d.validate()
    assert e.value.status == cb.Status.INVALID_VALUE


def test_reference_rns_frontend_binds_this_library():
    load_reference_package()
    spec = importlib.util.spec_from_file_location("ref_cubutterfly.rns", REF_PY / "rns.py")
    rns = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rns)
    rlib = rns.Library(str(cb.DEFAULT_LIBRARY))
    with pytest.raises(rns.Error) as e:
        rns.Plan(rlib, {"schema_version": 2})
    assert e.value.status == 1


def test_cli_reports_valid_and_invalid(tmp_path, lib):
    good = tmp_path / "good.json"
    with cb.Descriptor(lib, cb.Transform(op=cb.Operator.FFT, extents=[4096], batch=8)) as d:
        good.write_text(d.json())
    bad = tmp_path / "bad.json"
    bad.write_text('{"schema": "nope"}')
    r = subprocess.run([sys.executable, "-m", "cubutterfly_b200", str(good), str(bad), "--mappings", "2"],
                       capture_output=True, text=True, cwd=Path(__file__).resolve().parents[1])
    assert r.returncode == 1, r.stderr
    reports = [json.loads(line) for line in r.stdout.splitlines()]
    assert reports[0]["valid"] and len(reports[0]["mappings"]) >= 1
    assert not reports[1]["valid"] and "error" in reports[1]
