"""CPU: every Python file of the package, the tests, the oracle and the entry
scripts byte-compiles (scripts that only run under torchrun or on a GPU are not
imported by the other tests)."""
import os
import py_compile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_all_python_sources_compile(tmp_path):
    bad = []
    tops = ["kvmem_b200", "tests", "oracle"]
    walk = [(ROOT, [], [f for f in os.listdir(ROOT) if f.endswith(".py")])]
    for t in tops:
        for d, dirs, files in os.walk(os.path.join(ROOT, t)):
            dirs[:] = [x for x in dirs if not x.startswith((".", "_"))]
            walk.append((d, dirs, files))
    for d, _, files in walk:
        for f in files:
            if f.endswith(".py"):
                try:
                    py_compile.compile(os.path.join(d, f), cfile=str(tmp_path / "x.pyc"), doraise=True)
                except py_compile.PyCompileError as e:
                    bad.append(str(e))
    assert not bad, bad
