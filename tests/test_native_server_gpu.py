"""`vmc_run --serve`: the native OpenAI server over the GPU engine (csrc/server/ + the engine of
csrc/runtime/vmc_run.cpp). A greedy request must return the tokens the offline runtime produces for
the same prompt (same kernels, same steps: one prefill chunk, then decode steps replayed from the
batch-1 graph), decoded by the checkpoint's tokenizer; sampled, penalised and concurrent requests must
complete; the process must stop cleanly on SIGTERM. Request handling, streaming and scheduling of the
same server are covered on the CPU by tests/test_native_server_cpu.py."""
import http.client
import json
import os
import signal
import struct
import subprocess
import threading
import time

import numpy as np
import pytest

from vm_c_b200.gguf.random_init import preset, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource
from vm_c_b200.server.tokenizer import Tokenizer

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "vm_c_b200", "_ext", "runtime", "vmc_run")
ARGS = ["--max-num-seqs", "8", "--max-num-batched-tokens", "128", "--max-model-len", "256", "--num-blocks", "256"]


@pytest.fixture(scope="module")
def exe():
    if not os.path.exists(EXE):
        from vm_c_b200._build import build_runtime
        build_runtime()
    return EXE


def post(port, path, body):
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=120)
    c.request("POST", path, body=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    r = c.getresponse()
    out = r.status, json.loads(r.read())
    c.close()
    return out


def test_native_server_on_gpu(exe, tmp_path):
    cfg = preset("tiny-llama")
    path = str(tmp_path / "m.gguf")
    write_random_gguf(path, cfg, "Q8_0", seed=3)
    prompt = np.random.default_rng(9).integers(3, cfg.vocab, (1, 40)).astype(np.int32)
    pf = tmp_path / "p.bin"
    pf.write_bytes(struct.pack("<ii", *prompt.shape) + prompt.tobytes())
    dump = tmp_path / "t.json"
    r = subprocess.run([exe, path, "--prompts", str(pf), "--gen", "12", "--dump-tokens", str(dump)] + ARGS,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    offline = json.load(open(dump))[0]
    tok = Tokenizer.from_gguf(GgufSource(path))

    port_file = tmp_path / "port"
    proc = subprocess.Popen([exe, path, "--serve", "--port", "0", "--port-file", str(port_file)] + ARGS,
                            stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
    try:
        t0 = time.time()
        while not port_file.exists() or not port_file.read_text().strip():
            assert proc.poll() is None, proc.stderr.read().decode()[-2000:]
            assert time.time() - t0 < 240, "server did not start"
            time.sleep(0.1)
        port = int(port_file.read_text())
        st, out = post(port, "/v1/completions", {"prompt": prompt[0].tolist(), "max_tokens": 12, "temperature": 0,
                                                 "ignore_eos": True})
        assert st == 200, out
        assert out["usage"]["completion_tokens"] == 12
        assert out["choices"][0]["text"] == tok.decode(offline), (out, offline)
        # sampled, penalised and concurrent requests
        bodies = [{"prompt": prompt[0, : 10 + i].tolist(), "max_tokens": 12, "ignore_eos": True,
                   "temperature": 0.8, "top_p": 0.9, "seed": i} for i in range(6)]
        bodies.append({"prompt": prompt[0].tolist(), "max_tokens": 12, "ignore_eos": True,
                       "repetition_penalty": 1.3, "frequency_penalty": 0.5, "temperature": 0})
        res = [None] * len(bodies)

        def run(i):
            res[i] = post(port, "/v1/completions", bodies[i])
        th = [threading.Thread(target=run, args=(i,)) for i in range(len(bodies))]
        for t in th:
            t.start()
        for t in th:
            t.join(240)
        for st, out in res:
            assert st == 200 and out["usage"]["completion_tokens"] == 12, out
        # a seeded request served alone twice samples the same tokens
        a = post(port, "/v1/completions", bodies[2])[1]
        b = post(port, "/v1/completions", bodies[2])[1]
        assert a["choices"][0]["text"] == b["choices"][0]["text"]
        c = http.client.HTTPConnection("127.0.0.1", port, timeout=30)
        c.request("GET", "/health")
        assert json.loads(c.getresponse().read()) == {"status": "ok"}
        c.close()
    finally:
        proc.send_signal(signal.SIGTERM)
        try:
            rc = proc.wait(60)
        except subprocess.TimeoutExpired:
            proc.kill()
            rc = proc.wait()
    assert rc == 0, proc.stderr.read().decode()[-2000:]
