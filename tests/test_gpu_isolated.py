"""Runs the GPU tests of kernels that have not yet had a GPU run -- those
marked `isolated` -- each file in its own child pytest process, plus the
tree-attention tests under the opt-in 64-key kernel (MTP_ATTN_KERNEL=2).
A fault in one of them then cannot leave this process's CUDA context
unusable for the tests after it.  Each child must pass; until a first GPU
run has confirmed them, a failing child is reported as an expected failure
(non-strict xfail) with the end of its output."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.xfail(reason="first GPU run pending", strict=False)]

HERE = os.path.dirname(os.path.abspath(__file__))

# name -> (test files, extra environment, -k expression)
CHILDREN = {
    "streamk": (["test_gpu_streamk.py"], {}, None),
    "tall_tiles": (["test_gpu_tall_tiles.py"], {}, None),
    "tree_attn_rmsnorm_linear": (["test_gpu_tree_attn_rmsnorm_linear.py"], {}, None),
    "nccl_abi": (["test_gpu_nccl_abi.py"], {"NCCL_NVLS_ENABLE": "0"}, None),
    "exchange_single_gpu": (["test_gpu_exchange_single.py"], {}, None),
    "edge_shapes": (["test_gpu_edge_shapes.py"], {}, None),
    "attention_64key_kernel": (["test_gpu_attention_tc.py", "test_gpu_parity.py"], {"MTP_ATTN_KERNEL": "2"},
                               "attention or edge_cases or device_status"),
    # smaller operators and whole-path checks, one child for all of them
    "operators": (["test_verify_step.py", "test_paged_kv_write.py", "test_quant_attention_int4.py",
                   "test_gpu_sqattn.py", "test_gpu_graphs.py", "test_gpu_canary.py"], {}, None),
}


@pytest.mark.parametrize("name", sorted(CHILDREN))
def test_child(name):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    files, extra, kexpr = CHILDREN[name]
    env = dict(os.environ, MTP_ISOLATED_RUN="1", **extra)
    cmd = [sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider"]
    if kexpr:
        cmd += ["-k", kexpr]
    cmd += [os.path.join(HERE, f) for f in files]
    r = subprocess.run(cmd, env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=600)
    tail = "\n".join((r.stdout + r.stderr).strip().splitlines()[-40:])
    assert r.returncode == 0, f"child pytest for {name} exited {r.returncode}:\n{tail}"
