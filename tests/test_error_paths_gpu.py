"""The failure path of the device-side waits, made to run out without
faulting or hanging a GPU.

- One GPU: the tensor-parallel barrier kernel of a 2-rank exchange whose
  second rank is a buffer nothing writes (a flag nothing sets) must return
  within its short wait limit with the error flag set, and leave the GPU
  usable; with the peer's post in place the same kernel completes.
- Two GPUs, one process per rank: a rank that skips a step (between steps,
  with nothing of its own in flight) makes the other rank's decode wait run
  out after STRASGPT_WAIT_LIMIT_MS; that rank's host then stops with the
  reference's error convention ("[StrasGPT] Error ..." on stderr, exit
  status 1), as source/transformer.c's UTIL_DIE does (include/util.h:9-26
  of the reference). No NCCL, no NVLink multicast: gloo on the host and
  plain peer stores."""
import ctypes
import os
import subprocess
import sys
import textwrap
import time

import pytest

from conftest import model_dir
from strasgpt_b200 import configs, runtime

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _wait_check():
    L = runtime.lib()
    f = L.strasgpt_k_tp_wait_check
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def test_wait_check_rejects_bad_limits():
    # Host-side argument checks only: no device work.
    f = _wait_check()
    assert f(0, 0, None) == -1
    assert f(-5, 1, None) == -1
    assert f(600000, 0, None) == -1


@pytest.mark.gpu
def test_wait_that_runs_out_returns_an_error_status(cuda):
    torch = cuda
    f = _wait_check()
    t0 = time.time()
    assert f(100, 0, None) == 1          # nothing posts: the wait runs out
    assert time.time() - t0 < 10.0
    assert f(1000, 1, None) == 0         # the peer's post is there: completes
    # The context is still usable: a kernel after the timed-out one.
    L = runtime.lib()
    x = torch.randn(4, 256, device="cuda")
    w = torch.ones(256, device="cuda").to(torch.bfloat16).view(torch.int16)
    y = torch.empty_like(x)
    assert L.strasgpt_k_rmsnorm_rows(x.data_ptr(), 4, 256, w.data_ptr(), 1e-5, y.data_ptr(),
                                     None) == 0
    torch.cuda.synchronize()
    want = x / torch.sqrt((x * x).mean(dim=1, keepdim=True) + 1e-5)
    assert (y - want).abs().max().item() < 1e-5


RANK_SCRIPT = textwrap.dedent("""
    import datetime, os, sys, time
    sys.path.insert(0, {root!r})
    import numpy as np
    import torch.distributed as dist
    from strasgpt_b200 import Transformer, configs, synth
    rank = int(sys.argv[1])
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:{port}", rank=rank,
                            world_size=2, timeout=datetime.timedelta(seconds=60))
    cfg = configs.get("t_llama")
    m = Transformer({mdir!r}, rank=rank, world=2, device=rank)
    tok = int(np.argmax(m.predict(synth.prompt_tokens(cfg), 1)[0]))
    m.predict([tok], 1)                      # one decode step on both ranks
    dist.barrier()                           # both are between steps here
    if rank == 1:
        print("rank 1 skips the next step", flush=True)
        time.sleep(8)                        # stays alive while rank 0 waits
        os._exit(0)
    m.predict([tok], 1)                      # rank 1 never joins this step
    print("rank 0 returned from a step its peer skipped", flush=True)
""")


@pytest.mark.gpu
def test_rank_skipping_a_step_stops_the_other_with_an_error(cuda, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    script = tmp_path / "rank.py"
    script.write_text(RANK_SCRIPT.format(root=ROOT, port=port,
                                         mdir=model_dir(configs.get("t_llama"))))
    env = dict(os.environ, STRASGPT_WAIT_LIMIT_MS="300", NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(script), str(r)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in range(2)]
    outs = [p.communicate(timeout=300) for p in procs]
    assert procs[1].returncode == 0, outs[1][1][-2000:]
    assert procs[0].returncode == 1, outs[0]
    assert "[StrasGPT] Error" in outs[0][1], outs[0][1][-2000:]
    assert "timed out" in outs[0][1] or "did not post" in outs[0][1], outs[0][1][-2000:]
    assert "returned from a step" not in outs[0][0]
