"""Builds the native extensions in-tree.

Two extensions:
  * ``_host``  — C++17 host runtime (GGUF, quant codecs, block manager, scheduler). No CUDA.
  * ``_cuda``  — sm_100a kernels (tcgen05 / TMA GEMMs, attention, norms, sampling, comm) and their
                 launchers. Compiled only for ``sm_100a``; nothing else is generated.
and three executables:
  * ``vmc_run`` — the serving loop without Python or PyTorch (csrc/runtime/vmc_run.cpp): the same
                 kernels, native forward, scheduler and GGUF reader, linked against the CUDA runtime
                 and driver only; with ``--serve`` it is the native OpenAI-compatible server
                 (csrc/server/);
  * ``vmc_serve_cpu`` — the same server over a host-only rule backend instead of the GPU forward
                 (csrc/server/serve_cpu.cpp; run by tests/test_native_server_cpu.py);
  * ``vmc_tsan_stress`` — the host library (scheduler, block manager, quant codecs, BPE core) built
                 with ThreadSanitizer around a multi-threaded stress driver (csrc/host/tsan_stress.cpp;
                 run by tests/test_tsan_host.py, not part of build()).

The shared objects land in ``vm_c_b200/_ext/<name>/`` so that they travel with a copy of the
repository; :mod:`vm_c_b200._native` imports them from there without invoking the compiler.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
EXT_DIR = PKG_DIR / "_ext"
CSRC = REPO_DIR / "csrc"

HOST_SOURCES = ["host/gguf.cpp", "host/quants.cpp", "host/block_manager.cpp", "host/scheduler.cpp",
                "host/tokenizer.cpp", "host/turboquant.cpp", "host/safetensors.cpp", "host/bindings.cpp"]

SM100_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a"]


def cuda_sources() -> list[str]:
    kdir = CSRC / "kernels"
    return sorted(str(p) for p in kdir.glob("*.cu")) + sorted(str(p) for p in kdir.glob("*.cpp"))


def _jobs() -> None:
    os.environ.setdefault("MAX_JOBS", str(max(1, min(16, os.cpu_count() or 4))))


def build_host(verbose: bool = False):
    from torch.utils.cpp_extension import load
    _jobs()
    out = EXT_DIR / "host"
    out.mkdir(parents=True, exist_ok=True)
    return load(name="_host", sources=[str(CSRC / s) for s in HOST_SOURCES],
                extra_cflags=["-O3", "-std=c++17", "-fvisibility=hidden", "-Wno-unused-function"],
                extra_include_paths=[str(CSRC / "host")], build_directory=str(out), verbose=verbose,
                is_python_module=True)


def build_cuda(verbose: bool = False):
    from torch.utils.cpp_extension import load
    _jobs()
    out = EXT_DIR / "cuda"
    out.mkdir(parents=True, exist_ok=True)
    cuda_flags = SM100_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                                "-Xptxas=-v" if os.environ.get("VMC_PTXAS_VERBOSE") else "-Xptxas=-O3",
                                "-DNDEBUG", "-U__CUDA_NO_HALF_OPERATORS__",
                                "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
                                "-U__CUDA_NO_HALF2_OPERATORS__"] + os.environ.get("VMC_NVCC_EXTRA", "").split()
    return load(name="_cuda", sources=cuda_sources(),
                extra_cflags=["-O3", "-std=c++17"], extra_cuda_cflags=cuda_flags,
                extra_include_paths=[str(CSRC / "kernels"), str(CSRC / "host")],
                extra_ldflags=["-lcuda"], build_directory=str(out), verbose=verbose,
                is_python_module=True)


RUNTIME_HOST = ["host/gguf.cpp", "host/quants.cpp", "host/block_manager.cpp", "host/scheduler.cpp",
                "host/tokenizer.cpp"]
RUNTIME_EXCLUDE = {"ops.cpp"}   # the PyTorch bindings
SERVER_SOURCES = ["server/json.cpp", "server/unicode.cpp", "server/text_tokenizer.cpp", "server/jinja.cpp",
                  "server/chat.cpp", "server/http.cpp", "server/serve_loop.cpp", "server/openai.cpp"]
GEN_DIR = EXT_DIR / "gen"


def gen_unicode_ranges() -> Path:
    """Writes the letter / number / whitespace / mark code point ranges of the server's pre-tokenisers
    (csrc/server/unicode.cpp includes them), taken from the `regex` module that the Python tokenizer
    uses so that both split text identically."""
    out = GEN_DIR / "unicode_ranges.inc"
    version = "// unicode classes v2: letter 1, number 2, space 4, mark 8"
    if out.exists() and out.read_text().startswith(version):
        return out
    import regex
    chars = "".join(chr(c) for c in range(0x110000) if not 0xD800 <= c <= 0xDFFF)
    cls = bytearray(0x110000)
    for bit, pat in ((1, r"\p{L}+"), (2, r"\p{N}+"), (4, r"\s+"), (8, r"\p{M}+")):
        for m in regex.compile(pat).finditer(chars):
            for ch in m.group(0):
                cls[ord(ch)] |= bit
    rows, c = [], 0
    while c < 0x110000:
        if cls[c]:
            lo = c
            while c + 1 < 0x110000 and cls[c + 1] == cls[lo]:
                c += 1
            rows.append((lo, c, cls[lo]))
        c += 1
    GEN_DIR.mkdir(parents=True, exist_ok=True)
    lines = [version, "// Generated by vm_c_b200/_build.py gen_unicode_ranges(): {lo, hi, class bits}.",
             "const Range kRanges[] = {"]
    for k in range(0, len(rows), 4):
        lines.append("    " + " ".join("{0x%X, 0x%X, %d}," % r for r in rows[k:k + 4]))
    lines.append("};")
    tmp = out.with_suffix(".tmp")
    tmp.write_text("\n".join(lines) + "\n")
    tmp.replace(out)
    return out


def build_runtime(verbose: bool = False) -> Path:
    """Compile and link vm_c_b200/_ext/runtime/vmc_run (objects are rebuilt when their source or a
    header in csrc/ is newer)."""
    import concurrent.futures
    import shutil
    import subprocess
    out = EXT_DIR / "runtime"
    obj = out / "obj"
    obj.mkdir(parents=True, exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    kdir = CSRC / "kernels"
    srcs = [p for p in sorted(kdir.glob("*.cu")) + sorted(kdir.glob("*.cpp")) if p.name not in RUNTIME_EXCLUDE]
    srcs += [CSRC / s for s in RUNTIME_HOST + SERVER_SOURCES] + [CSRC / "runtime" / "vmc_run.cpp"]
    gen_unicode_ranges()
    headers = max(p.stat().st_mtime for p in CSRC.rglob("*") if p.suffix in (".h", ".hpp", ".cuh", ".inc"))
    flags = SM100_FLAGS + ["-O3", "-std=c++17", "--expt-relaxed-constexpr", "-lineinfo", "-DNDEBUG",
                           f"-I{kdir}", f"-I{CSRC / 'host'}", f"-I{CSRC / 'server'}", f"-I{GEN_DIR}",
                           "-Xcompiler", "-fPIC"]

    def compile_one(src: Path) -> Path:
        o = obj / (src.parent.name + "_" + src.name + ".o")
        if not o.exists() or o.stat().st_mtime < max(src.stat().st_mtime, headers):
            cmd = [nvcc] + flags + ["-x", "cu" if src.suffix == ".cu" else "c++", "-c", str(src), "-o", str(o)]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr[-4000:]}")
            if verbose:
                print("compiled", src.name)
        return o

    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(16, os.cpu_count() or 4))) as ex:
        objs = list(ex.map(compile_one, srcs))
    exe = out / "vmc_run"
    r = subprocess.run([nvcc] + SM100_FLAGS + [str(o) for o in objs] + ["-o", str(exe), "-lcuda", "-lpthread"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link of vmc_run failed:\n{r.stderr[-4000:]}")
    return exe


SERVE_CPU_HOST = ["host/gguf.cpp", "host/block_manager.cpp", "host/scheduler.cpp", "host/tokenizer.cpp"]


def build_serve_cpu(verbose: bool = False, tsan: bool = False) -> Path:
    """Compile and link vm_c_b200/_ext/serve/vmc_serve_cpu with the host compiler (objects are rebuilt
    when their source or a header in csrc/ is newer). tsan=True builds vm_c_b200/_ext/tsan/vmc_serve_cpu
    with ThreadSanitizer instead (HTTP threads, serving loop and streams checked for data races)."""
    import concurrent.futures
    import shutil
    import subprocess
    out = EXT_DIR / ("tsan" if tsan else "serve")
    obj = out / ("serve_obj" if tsan else "obj")
    obj.mkdir(parents=True, exist_ok=True)
    gen_unicode_ranges()
    cxx = shutil.which("g++") or "c++"
    srcs = [CSRC / s for s in SERVE_CPU_HOST + SERVER_SOURCES + ["server/serve_cpu.cpp"]]
    headers = max(p.stat().st_mtime for p in list(CSRC.rglob("*")) + [GEN_DIR / "unicode_ranges.inc"]
                  if p.suffix in (".h", ".hpp", ".inc"))
    flags = ["-O2", "-std=c++17", "-pthread", "-Wall", f"-I{CSRC / 'host'}", f"-I{CSRC / 'server'}", f"-I{GEN_DIR}"]
    if tsan:
        flags = ["-O1", "-g", "-fsanitize=thread"] + flags[1:]

    def compile_one(src: Path) -> Path:
        o = obj / (src.parent.name + "_" + src.name + ".o")
        if not o.exists() or o.stat().st_mtime < max(src.stat().st_mtime, headers):
            r = subprocess.run([cxx] + flags + ["-c", str(src), "-o", str(o)], capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"g++ failed on {src}:\n{r.stderr[-4000:]}")
            if verbose:
                print("compiled", src.name)
        return o

    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(16, os.cpu_count() or 4))) as ex:
        objs = list(ex.map(compile_one, srcs))
    exe = out / "vmc_serve_cpu"
    if not exe.exists() or exe.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        r = subprocess.run([cxx, "-pthread"] + (["-fsanitize=thread"] if tsan else []) + [str(o) for o in objs] +
                           ["-o", str(exe)], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link of vmc_serve_cpu failed:\n{r.stderr[-4000:]}")
    return exe


TSAN_HOST = ["host/scheduler.cpp", "host/block_manager.cpp", "host/quants.cpp", "host/tokenizer.cpp",
             "host/tsan_stress.cpp"]


def build_tsan(verbose: bool = False) -> Path:
    """Compile vm_c_b200/_ext/tsan/vmc_tsan_stress with -fsanitize=thread (rebuilt when a host source
    or header is newer than the executable)."""
    import shutil
    import subprocess
    out = EXT_DIR / "tsan"
    out.mkdir(parents=True, exist_ok=True)
    exe = out / "vmc_tsan_stress"
    srcs = [CSRC / s for s in TSAN_HOST]
    newest = max(p.stat().st_mtime for p in srcs + list((CSRC / "host").glob("*.hpp")))
    if exe.exists() and exe.stat().st_mtime >= newest:
        return exe
    cxx = shutil.which("g++") or "c++"
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-pthread", f"-I{CSRC / 'host'}"] + \
        [str(p) for p in srcs] + ["-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ThreadSanitizer build failed:\n{r.stderr[-4000:]}")
    if verbose:
        print("built", exe)
    return exe


def build_protocol_sim(verbose: bool = False) -> Path:
    """Compile vm_c_b200/_ext/tsan/vmc_tp_protocol_sim (csrc/host/tp_protocol_sim.cpp) with
    ThreadSanitizer: the tensor-parallel flag protocol with ranks and CTAs as threads."""
    import shutil
    import subprocess
    out = EXT_DIR / "tsan"
    out.mkdir(parents=True, exist_ok=True)
    exe = out / "vmc_tp_protocol_sim"
    src = CSRC / "host" / "tp_protocol_sim.cpp"
    if exe.exists() and exe.stat().st_mtime >= src.stat().st_mtime:
        return exe
    cxx = shutil.which("g++") or "c++"
    r = subprocess.run([cxx, "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-pthread", str(src), "-o", str(exe)],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"protocol simulation build failed:\n{r.stderr[-4000:]}")
    if verbose:
        print("built", exe)
    return exe


def build_all(verbose: bool = False) -> None:
    build_host(verbose)
    build_cuda(verbose)
    build_runtime(verbose)
    build_serve_cpu(verbose)


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    v = "-v" in sys.argv
    if what in ("host", "all"):
        build_host(v)
    if what in ("cuda", "all"):
        build_cuda(v)
    if what in ("runtime", "all"):
        build_runtime(v)
    if what in ("serve", "all"):
        build_serve_cpu(v)
    if what == "tsan":
        build_tsan(v)
        build_protocol_sim(v)
