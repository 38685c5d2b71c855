"""The native host library under ThreadSanitizer (csrc/host/tsan_stress.cpp): producer threads feeding
one scheduler owner through a command queue, independent schedulers on several threads compared
with lone runs, the multi-threaded quant codecs, and a BPE core shared by encoding threads. Any data
race ThreadSanitizer reports fails the run (exit status 66), as does any failed check. CPU only."""
import os
import shutil
import subprocess

import pytest

from vm_c_b200._build import build_tsan


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++ with ThreadSanitizer")
def test_host_library_is_race_free_under_tsan():
    exe = build_tsan()
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66 second_deadlock_stack=1")
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, (r.returncode, r.stdout[-2000:], r.stderr[-6000:])
    assert r.stdout.strip().splitlines()[-1] == "ok", r.stdout
    assert "WARNING: ThreadSanitizer" not in r.stderr, r.stderr[-6000:]
