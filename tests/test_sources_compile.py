"""CPU: every Python file of the repository byte-compiles (scripts that only run
under torchrun or on a GPU are not imported by the other tests)."""
import os
import py_compile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_all_python_sources_compile(tmp_path):
    bad = []
    for d, dirs, files in os.walk(ROOT):
        dirs[:] = [x for x in dirs if not x.startswith(".") and x not in ("_work", "gpurun_out", "baseline", "_ref")]
        for f in files:
            if f.endswith(".py"):
                try:
                    py_compile.compile(os.path.join(d, f), cfile=str(tmp_path / "x.pyc"), doraise=True)
                except py_compile.PyCompileError as e:
                    bad.append(str(e))
    assert not bad, bad
