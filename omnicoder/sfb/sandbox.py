"""Code sandboxes for program-aided checks (reference src/omnicoder/sfb/runtime/sandbox.py:1-108):
run a candidate program with its tests and report pass / fail with the captured output.

  PythonSandbox   `python -I` (isolated mode: no user site, no environment hooks) in a fresh
                  temporary directory, wall-clock timeout, and on Linux CPU-time, address-space
                  and file-size limits applied in the child before it starts;
  CppSandbox      g++ -O2 -std=c++17 then the binary, same limits;
  HTTPSandbox     POST {"code", "tests", "timeout"} to a remote runner, which answers
                  {"ok", "stdout", "stderr"};
  verify_with_tests  the solution as `solution.py` beside a pytest file, pytest run under the same
                  limits (plugins not auto-loaded), with the passed / failed / error counts
                  (reference src/omnicoder/tools/code_verifier.py:1-97; a failing pytest run is
                  the answer here, not a reason to fall back to executing the test file, which would
                  only define the test functions and exit 0).
The tests run after the code; the run passes when the process exits 0 (Python: and printed the
end marker, so a test file that exits early does not pass).  This isolates resources, not
privileges: the child runs as the calling user, so it is meant for model-written snippets under
test, not for adversarial code.
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile
from dataclasses import dataclass

_MARK = "__omnicoder_sandbox_ok__"


@dataclass
class SandboxResult:
    ok: bool
    stdout: str
    stderr: str
    returncode: int | None = None


def _limits(cpu_s: int, mem_bytes: int):
    def apply():
        try:
            import resource
            resource.setrlimit(resource.RLIMIT_CPU, (cpu_s, cpu_s))
            resource.setrlimit(resource.RLIMIT_AS, (mem_bytes, mem_bytes))
            resource.setrlimit(resource.RLIMIT_FSIZE, (16 << 20, 16 << 20))
        except (ImportError, ValueError, OSError):
            pass
    return apply if os.name == "posix" else None


def _run(args, cwd, timeout, mem_bytes, env_extra: dict | None = None) -> SandboxResult:
    env = {"PATH": os.environ.get("PATH", "/usr/bin:/bin"), "LANG": "C.UTF-8", **(env_extra or {})}
    try:
        p = subprocess.run(args, cwd=cwd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                           timeout=max(1, timeout), preexec_fn=_limits(max(1, timeout), mem_bytes), env=env)
        return SandboxResult(p.returncode == 0, p.stdout, p.stderr, p.returncode)
    except subprocess.TimeoutExpired as e:
        out = e.stdout.decode() if isinstance(e.stdout, bytes) else (e.stdout or "")
        return SandboxResult(False, out, "timeout", None)


class PythonSandbox:
    def __init__(self, python: str | None = None, mem_bytes: int = 4 << 30):
        self.python, self.mem = python or sys.executable, mem_bytes

    def run(self, code: str, tests: str = "", timeout: int = 5) -> SandboxResult:
        body = "\n".join("    " + line for line in (tests or "pass").splitlines())
        src = f"{code}\n\nif __name__ == '__main__':\n{body}\n    print({_MARK!r})\n"
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "main.py")
            with open(path, "w", encoding="utf-8") as f:
                f.write(src)
            r = _run([self.python, "-I", path], td, timeout, self.mem)
        r.ok = r.ok and _MARK in r.stdout
        r.stdout = r.stdout.replace(_MARK + "\n", "")
        return r


class CppSandbox:
    def __init__(self, cxx: str = "g++", mem_bytes: int = 4 << 30):
        self.cxx, self.mem = cxx, mem_bytes

    def run(self, code: str, tests: str = "", timeout: int = 10) -> SandboxResult:
        with tempfile.TemporaryDirectory() as td:
            src, exe = os.path.join(td, "main.cpp"), os.path.join(td, "a.out")
            with open(src, "w", encoding="utf-8") as f:
                f.write(f"{code}\n\nint main() {{\n{tests}\nreturn 0;\n}}\n")
            b = _run([self.cxx, src, "-O2", "-std=c++17", "-o", exe], td, timeout, 4 << 30)
            if not b.ok:
                return b
            return _run([exe], td, timeout, self.mem)


class HTTPSandbox:
    def __init__(self, url: str):
        self.url = url

    def run(self, code: str, tests: str = "", timeout: int = 5) -> SandboxResult:
        import requests
        try:
            r = requests.post(self.url, json={"code": code, "tests": tests, "timeout": timeout}, timeout=timeout + 5)
            d = r.json()
            return SandboxResult(bool(d.get("ok")), str(d.get("stdout", "")), str(d.get("stderr", "")))
        except Exception as e:
            return SandboxResult(False, "", f"remote sandbox error: {e}")


@dataclass
class VerifyReport:
    ok: bool
    passed: int
    failed: int
    errors: int
    returncode: int | None
    log: str


def verify_with_tests(code: str, tests: str, tests_name: str = "test_solution.py", timeout: int = 30,
                      mem_bytes: int = 4 << 30, python: str | None = None) -> VerifyReport:
    import re
    if not tests_name.startswith("test_") or not tests_name.endswith(".py"):
        raise ValueError("tests_name must look like test_*.py so that pytest collects it")
    with tempfile.TemporaryDirectory() as td:
        with open(os.path.join(td, "solution.py"), "w", encoding="utf-8") as f:
            f.write(code)
        with open(os.path.join(td, tests_name), "w", encoding="utf-8") as f:
            f.write(tests)
        r = _run([python or sys.executable, "-I", "-m", "pytest", "-q", "-p", "no:cacheprovider", tests_name], td,
                 timeout, mem_bytes, {"PYTEST_DISABLE_PLUGIN_AUTOLOAD": "1", "PYTHONPATH": td})
    out = r.stdout + "\n" + r.stderr

    def count(word):
        m = re.findall(rf"(\d+) {word}", out)
        return int(m[-1]) if m else 0
    passed, failed, errors = count("passed"), count("failed"), count("errors?")
    return VerifyReport(r.returncode == 0 and passed > 0 and failed == 0 and errors == 0, passed, failed, errors,
                      r.returncode, out[-20000:])
