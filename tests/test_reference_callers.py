"""The reference's callers, unchanged, drive this repository's kernels (the drop-in claim).

Each case runs baseline/ref_callers.py in a fresh process whose import path holds this
package and the reference installed by baseline/install_reference.py (baseline/_ref), so the
reference's bench/attention.py, model/bd3lm.py, sample/sampler.py, inference/generate.py,
bench/attention_bench.py and train/train.py import ``kernels`` from here. Skipped when the
reference has not been installed.

Tolerances: the "custom" backend is the reference's own masked attention with fp32 logits on
bf16 inputs under autocast; "bsfa" / "split_kv" / "bsdfa" are the bf16 kernels, so their
outputs differ from it by bf16 rounding of P and O (north_star's 2e-2 on attention outputs),
which the model carries into its log-probabilities and gradients.
"""

import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

RUNNER = os.path.join(REPO, "baseline", "ref_callers.py")
REF = os.path.join(REPO, "baseline", "_ref")

pytestmark = pytest.mark.skipif(
    not os.path.isdir(os.path.join(REF, "model")),
    reason="reference not installed (python baseline/install_reference.py --src <checkout>)")


def run_case(name: str, args: dict | None = None, timeout: int = 900) -> dict:
    cmd = [sys.executable, RUNNER, name] + ([json.dumps(args)] if args else [])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=REPO)
    assert r.returncode == 0, f"{name} failed:\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    return json.loads(line)


def test_reference_registry_binds_this_kernels_package():
    out = run_case("registry")
    assert out["registry_file"] == os.path.join("baseline", "_ref", "bench", "attention.py")
    assert out["kernels_from"] == os.path.join("diffusion-llm_b200", "kernels")
    assert {"custom", "bsfa", "bsdfa", "split_kv"} <= set(out["backends"])


@pytest.mark.gpu
def test_bd3lm_forward_backward_bsfa_matches_custom():
    out = run_case("train")
    assert out["masked_equal"]
    assert out["loss_rel"] < 1e-2, out
    assert out["prob_max_abs"] < 2e-2, out
    assert out["grad_rel_norm"] < 3e-2, out


@pytest.mark.gpu
def test_sample_bd3lm_split_kv_matches_custom():
    out = run_case("sample")
    assert out["tokens_shape"] == [2, 64] and out["no_mask_left"]
    assert out["cached_logprob_max_abs"] < 5e-2, out
    assert out["uncached_logprob_max_abs"] < 5e-2, out
    assert out["cached_vs_uncached_max_abs"] < 5e-2, out
    # the draws are the same uniforms; near-ties of the Gumbel-max may flip a token, after
    # which later blocks are conditioned on different text
    assert out["token_agreement"] >= 0.5, out


@pytest.mark.gpu
def test_generate_compile_rungs_trace_without_graph_breaks():
    out = run_case("compile")
    assert out["graph_breaks"] == {}, out
    assert out["library_decode_calls"] > 0, out
    assert out["tokens_shape"] == [1, 96 + 48] and out["no_mask_left"]
    assert out["compiled_vs_eager_logprob_max_abs"] < 5e-2, out


@pytest.mark.gpu
def test_attention_bench_runs_bsfa():
    out = run_case("attention_bench")
    assert out["check_passed"], out
    assert out["fwd_ms"] > 0 and out["bwd_ms"] > 0


@pytest.mark.gpu
def test_train_loop_bsfa_tracks_custom():
    out = run_case("train_loop")
    lb, lc = out["bsfa"]["losses"], out["custom"]["losses"]
    assert len(lb) == len(lc) == 24
    assert lb[-1] < lb[0] and lc[-1] < lc[0], out
    assert out["loss_max_rel_diff"] < 3e-2, out
