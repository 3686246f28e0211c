"""The drop-in boundary end to end: the reference's own command-line
program (source/strasgpt.c with its options, tokenizer and sampler, built
by oracle/Makefile) linked against libstrasgpt.so instead of the reference
forward pass, must print exactly the same greedy text as the same program
built on the reference's CPU forward pass, for the same model directory and
prompt. This exercises the C ABI as strasgpt.c uses it: the safetensors
reader, transformer_from_safetensors, transformer_logits_malloc, and
transformer_predict called from every thread of an OpenMP team."""
import os
import subprocess

import pytest

from conftest import model_dir
from strasgpt_b200 import configs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPU = os.path.join(ROOT, "oracle", "_ref", "strasgpt_cpu")
GPU = os.path.join(ROOT, "oracle", "_ref", "strasgpt_gpu")
PROMPT = "Once upon a time, in a land far away"


def _generate(binary, mdir, steps, **extra_env):
    env = dict(os.environ, OMP_NUM_THREADS="4", **extra_env)
    r = subprocess.run([binary, "-m", mdir, "-n", str(steps), "-p", PROMPT, "--temp", "0",
                        "-t", "4"], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, f"{os.path.basename(binary)} failed: {r.stderr[-2000:]}"
    return r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["t_llama", "t_qwen", "t_untied", "t_gqa8"])
def test_reference_cli_on_the_gpu_library(cuda, name):
    if not (os.path.exists(CPU) and os.path.exists(GPU)):
        pytest.skip("reference CLI binaries not built (oracle/Makefile)")
    mdir = model_dir(configs.get(name))
    steps = 16
    want = _generate(CPU, mdir, steps)
    got = _generate(GPU, mdir, steps)
    assert want.strip(), "empty reference output"
    assert got == want


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["t_llama", "t_gqa8"])
def test_reference_cli_tensor_parallel_in_one_process(cuda, name):
    """The unmodified strasgpt.c on 2 GPUs: STRASGPT_NGPU=2 makes
    transformer_from_safetensors build a 2-rank group in the process."""
    if not (os.path.exists(CPU) and os.path.exists(GPU)):
        pytest.skip("reference CLI binaries not built (oracle/Makefile)")
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mdir = model_dir(configs.get(name))
    want = _generate(CPU, mdir, 16)
    got = _generate(GPU, mdir, 16, STRASGPT_NGPU="2")
    assert want.strip(), "empty reference output"
    assert got == want
