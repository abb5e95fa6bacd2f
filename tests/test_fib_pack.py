"""flashinfer-bench packaging (CPU): the Solution JSON of each operator, its
round trip through unpack, and that the packed sources compile on their own
(kernel.py's nvcc build, no GPU) into a library exporting the entry points."""
import ctypes
import importlib.util
import json

import pytest

from tests.conftest import submodule

pack = submodule("fib.pack")


def test_solution_fields():
    for which, definition, entry in (
            ("attention", "dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64", "kernel.py::launch_sparse_attention_c"),
            ("indexer", "dsa_topk_indexer_fp8_h64_d128_topk2048_ps64", "kernel.py::launch_topk_c")):
        s = pack.solution(which)
        assert s["definition"] == definition
        spec = s["spec"]
        assert spec["language"] == "python" and spec["entry_point"] == entry
        assert spec["target_hardware"] == ["NVIDIA_B200"] and spec["destination_passing_style"] is True
        paths = [x["path"] for x in s["sources"]]
        assert paths[0] == "kernel.py" and len(set(paths)) == len(paths)
        assert set(paths) == set(pack.FILES)
        json.dumps(s)   # serialisable
    with pytest.raises(ValueError):
        pack.solution("moe")


def test_unpack_round_trip(tmp_path):
    out = pack.write("attention", str(tmp_path / "json"))
    with open(out) as f:
        sol = json.load(f)
    files = pack.unpack(sol, str(tmp_path / "sol"))
    for p in files:
        rel = p[len(str(tmp_path / "sol")) + 1:]
        with open(p) as a, open(pack.FILES[rel]) as b:
            assert a.read() == b.read()
    bad = {"sources": [{"path": "../evil.py", "content": ""}]}
    with pytest.raises(ValueError):
        pack.unpack(bad, str(tmp_path / "sol2"))


def test_packed_sources_compile_alone(tmp_path, monkeypatch):
    """The unpacked solution builds with its own kernel.py (nvcc for sm_100a
    into $DSA_FIB_CACHE) and the library exports both entry points."""
    sol_dir = tmp_path / "sol"
    pack.unpack(pack.solution("indexer"), str(sol_dir))
    monkeypatch.setenv("DSA_FIB_CACHE", str(tmp_path / "cache"))
    spec = importlib.util.spec_from_file_location("dsa_fib_kernel_cpu", str(sol_dir / "kernel.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    lib_path = mod.build()
    assert lib_path.startswith(str(tmp_path / "cache"))
    assert mod.build() == lib_path   # cached by source hash
    lib = ctypes.CDLL(lib_path)
    for sym in ("dsa_sparse_attention_fwd", "dsa_sparse_attention_workspace_size", "dsa_topk_indexer_fwd",
                "dsa_topk_indexer_workspace_size", "dsa_status_string"):
        assert hasattr(lib, sym)
