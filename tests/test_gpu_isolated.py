"""Runs the GPU tests marked `isolated` -- each group of files in its own
child pytest process.  A fault in one of them then cannot leave
this process's CUDA context unusable for the tests after it.  Every child
must pass: a failing child fails this test, and its failing test ids are
printed on one line (`FAILED-IN-CHILD <name>: id, id, ...`) so they survive
the end of a long log."""

import os
import re
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu]

HERE = os.path.dirname(os.path.abspath(__file__))

# name -> (test files, extra environment, -k expression)
CHILDREN = {
    "streamk": (["test_gpu_streamk.py"], {}, None),
    "tree_attn_rmsnorm_linear": (["test_gpu_tree_attn_rmsnorm_linear.py"], {}, None),
    "nccl_abi": (["test_gpu_nccl_abi.py"], {"NCCL_NVLS_ENABLE": "0"}, None),
    "exchange_single_gpu": (["test_gpu_exchange_single.py"], {}, None),
    "edge_shapes": (["test_gpu_edge_shapes.py"], {}, None),
    "verify_step": (["test_verify_step.py"], {}, None),
    "paged_kv_write": (["test_paged_kv_write.py"], {}, None),
    "quant_attention_int4": (["test_quant_attention_int4.py"], {}, None),
    "sqattn": (["test_gpu_sqattn.py"], {}, None),
    "graphs": (["test_gpu_graphs.py"], {}, None),
    "canary": (["test_gpu_canary.py"], {}, None),
}


def failing_ids(output):
    """Test ids from pytest's short summary (`FAILED path::id - msg`, `ERROR ...`)."""
    ids = []
    for line in output.splitlines():
        m = re.match(r"^(FAILED|ERROR) (\S+)", line)
        if m:
            ids.append(m.group(2))
    return ids


@pytest.mark.parametrize("name", sorted(CHILDREN))
def test_child(name):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    files, extra, kexpr = CHILDREN[name]
    env = dict(os.environ, MTP_ISOLATED_RUN="1", **extra)
    cmd = [sys.executable, "-m", "pytest", "-q", "-rfE", "--tb=short", "-m", "gpu", "-p", "no:cacheprovider"]
    if kexpr:
        cmd += ["-k", kexpr]
    cmd += [os.path.join(HERE, f) for f in files]
    r = subprocess.run(cmd, env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    if r.returncode != 0:
        print(f"FAILED-IN-CHILD {name}: " + (", ".join(failing_ids(out)) or f"exit {r.returncode}"), flush=True)
    tail = "\n".join(out.strip().splitlines()[-40:])
    assert r.returncode == 0, f"child pytest for {name} exited {r.returncode}:\n{tail}"
