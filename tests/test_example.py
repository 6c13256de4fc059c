"""The example driver runs as a user would run it: one process, then two
ranks under torchrun, with a checkpoint written, resumed and continued.

CPU and gloo only (``MINISPEED_DEVICE=cpu``), small model and few steps.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SCRIPT = str(ROOT / "examples" / "train_lm.py")


def _env():
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")}
    env.update(MINISPEED_DEVICE="cpu", MINISPEED_BACKEND="gloo", CUDA_VISIBLE_DEVICES="",
               MINISPEED_PG_TIMEOUT_S="120", OMP_NUM_THREADS="2")
    return env


def _run(args, timeout=300):
    r = subprocess.run(args, cwd=ROOT, env=_env(), capture_output=True, text=True,
                       timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return r.stdout


SMALL = ["--dtype", "fp32", "--n-layer", "1", "--n-embd", "32", "--n-head", "2",
         "--block-size", "16", "--batch-size", "4", "--gas", "2", "--warmup", "2"]


def test_single_process_train_save_resume(tmp_path):
    out = tmp_path / "ckpt"
    log = _run([sys.executable, SCRIPT, *SMALL, "--zero", "2", "--steps", "4",
                "--log-every", "2", "--save-every", "2", "--ckpt-dir", str(out)])
    assert "step     1/4" in log and "step     4/4" in log
    assert "done:" in log and "sample:" in log
    assert (out / "latest").read_text() == "global_step4"
    assert sorted(os.listdir(out)) == ["global_step2", "global_step4", "latest"]

    log = _run([sys.executable, SCRIPT, *SMALL, "--zero", "2", "--steps", "6",
                "--log-every", "2", "--save-every", "0", "--ckpt-dir", str(out),
                "--resume", str(out)])
    assert "resumed" in log and "at step 4" in log
    assert "step     6/6" in log and "step     2/" not in log
    assert (out / "latest").read_text() == "global_step6"

    # an explicit dir/tag resumes that tag
    log = _run([sys.executable, SCRIPT, *SMALL, "--zero", "2", "--steps", "3",
                "--log-every", "1", "--save-every", "0", "--ckpt-dir", str(tmp_path / "b"),
                "--resume", str(out / "global_step2")])
    assert "at step 2" in log and "step     3/3" in log

    # so does the latest file itself
    log = _run([sys.executable, SCRIPT, *SMALL, "--zero", "2", "--steps", "7",
                "--log-every", "1", "--save-every", "0", "--ckpt-dir", str(tmp_path / "d"),
                "--resume", str(out / "latest")])
    assert "at step 6" in log and "step     7/7" in log


def test_json_config(tmp_path):
    log = _run([sys.executable, SCRIPT, "--config", str(ROOT / "examples" / "ds_config_tiny.json"),
                "--n-layer", "1", "--n-embd", "32", "--n-head", "2", "--block-size", "16",
                "--steps", "2", "--log-every", "1", "--save-every", "0",
                "--ckpt-dir", str(tmp_path / "c")])
    assert "step     2/2" in log and "done:" in log


@pytest.mark.parametrize("zero", [1, 3])
def test_two_ranks_under_torchrun(zero, tmp_path):
    from tests.helpers import free_port
    out = tmp_path / "ckpt"
    log = _run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                "--master-port", str(free_port()), SCRIPT, *SMALL, "--zero", str(zero),
                "--steps", "3", "--log-every", "1", "--save-every", "0",
                "--ckpt-dir", str(out)])
    assert "world=2" in log and "step     3/3" in log and "done:" in log
    names = sorted(os.listdir(out / "global_step3"))
    assert names == ["mp_rank_00_model_states.pt",
                     "zero_pp_rank0_mp_rank_00_optim_states.pt",
                     "zero_pp_rank1_mp_rank_00_optim_states.pt"]


def test_llama_arch(tmp_path):
    log = _run([sys.executable, SCRIPT, "--arch", "llama", "--dtype", "fp32", "--zero", "3",
                "--n-layer", "1", "--n-embd", "32", "--n-head", "4", "--n-kv-head", "2",
                "--block-size", "16", "--batch-size", "4", "--gas", "1", "--steps", "3",
                "--log-every", "1", "--save-every", "0", "--ckpt-dir", str(tmp_path / "l")])
    assert "step     3/3" in log and "sample:" in log
