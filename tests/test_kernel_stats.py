"""Compiled-kernel resources on the host: ptxas's report of a real sm_100a build, the B200 residency
it allows, the ABI/limit checks of the Backend protocol (check_abi, pipeline_stats, the validation
filters), compiler-line mapping through assemble, and the evaluator refusing a launch whose entry
was never compiled before anything reaches a GPU."""

from __future__ import annotations

import subprocess
from types import SimpleNamespace

import pytest

from shapeforge_b200 import kernel_stats as ks
from shapeforge_b200 import track_factory as tf
from shapeforge_b200.backend import CudaBackend, LaunchStage
from shapeforge_b200.build import nvcc
from shapeforge_b200.candidates import kernel_resources

SRC = r'''
extern "C" __global__ void staged(const float* x, float* y) {
    __shared__ float s[1024];
    s[threadIdx.x] = x[threadIdx.x];
    __syncthreads();
    y[threadIdx.x] = s[1023 - threadIdx.x];
}
extern "C" __global__ void plain(int* y, int n) { for (int i = 0; i < n; ++i) y[i] += i; }
'''


def test_ptxas_report_of_a_real_build():
    res = kernel_resources(SRC, name="kstats", use_cache=False)
    assert set(res) == {"staged", "plain"}
    assert res["staged"].static_smem == 4096 and res["staged"].barriers == 1
    assert res["plain"].static_smem == 0 and 0 < res["plain"].registers <= 255
    assert kernel_resources(SRC, name="kstats") == res  # the record beside the cached cubin


def test_parse_ignores_non_entry_lines():
    text = """ptxas info    : 0 bytes gmem
ptxas info    : Function properties for helper
    8 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Compiling entry function 'k' for 'sm_100a'
ptxas info    : Function properties for k
    16 bytes stack frame, 4 bytes spill stores, 8 bytes spill loads
ptxas info    : Used 40 registers, used 2 barriers, 512 bytes smem
"""
    assert ks.parse_ptxas(text) == {"k": ks.KernelResources("k", 40, 512, 16, 4, 8, 2)}


@pytest.mark.parametrize("regs,threads,smem,ctas,limit", [
    (32, 256, 0, 8, "registers"),      # 64K / (32*256) = 8 CTAs, the same as the 2048-thread bound
    (64, 1024, 0, 1, "registers"),
    (65, 1024, 0, 0, "registers"),     # 72 regs/thread after the 256-per-warp rounding: does not fit
    (16, 128, 100 * 1024, 2, "shared_memory"),
    (16, 32, 0, 32, "ctas"),
])
def test_residency(regs, threads, smem, ctas, limit):
    occ = ks.resident_ctas(ks.KernelResources("k", regs), threads, smem)
    assert occ["ctas"] == ctas and occ["limit"] == limit


def test_stage_checks_and_stats():
    res = {"k": ks.KernelResources("k", 40, 2048, spill_stores=8)}
    ok = LaunchStage("k", (296, 1, 1), (256, 1, 1), 0)
    assert ks.check_stages(res, [ok]) == []
    assert "was not compiled" in ks.check_stages(res, [LaunchStage("gone", (1, 1, 1), (32, 1, 1))])[0]
    assert "above the per-CTA limit" in ks.check_stages(res, [LaunchStage("k", (1, 1, 1), (32, 1, 1), 231 * 1024)])[0]
    assert "1025 threads" in ks.check_stages(res, [LaunchStage("k", (1, 1, 1), (1025, 1, 1))])[0]
    fat = {"k": ks.KernelResources("k", 128)}
    assert "do not fit one SM" in ks.check_stages(fat, [LaunchStage("k", (1, 1, 1), (1024, 1, 1))])[0]
    st = CudaBackend().pipeline_stats(res["k"], ok, {"sm_count": 148})
    assert st["thread_execution_width"] == 32 and st["launch_threadgroups"] == 296
    assert st["resident_ctas_per_sm"] == 6 and st["waves"] == pytest.approx(296 / (6 * 148))
    assert any("spill" in h for h in st["hints"])
    many = CudaBackend().pipeline_stats_many([(res["k"], ok), (fat["k"], LaunchStage("k", (64, 1, 1), (128, 1, 1)))], {})
    assert len(many["stages"]) == 2 and many["registers_per_thread"] == 128 and many["launch_threadgroups"] == 64
    assert any("SMs idle" in h for h in many["hints"])


def test_check_abi_uses_target_limits_and_validation_filter():
    b = CudaBackend()
    target = SimpleNamespace(id="b200", limits=SimpleNamespace(max_threads_per_threadgroup=1024,
                                                               max_threadgroup_memory_bytes=48 * 1024))
    kernels = [ks.KernelResources("k", 32, 64 * 1024)]
    stage = LaunchStage("k", (1, 1, 1), (128, 1, 1))
    problems = b.check_abi(None, kernels, target=target, spec=[stage])
    assert len(problems) == 1 and b.is_instrumented_size_only(problems)
    assert b.validation_problems(problems, [1024], 48 * 1024) == []
    assert b.validation_problems(problems, [64 * 1024], 48 * 1024) == problems
    assert b.check_abi(None, kernels, target=target, spec=[stage], device_info={"max_smem_per_block_optin": 232448}) == problems
    assert b.check_abi(None, [ks.KernelResources("k", 32, 1024)], target=target, spec=[stage]) == []
    assert b.validation_summary(size_only=False, target=target) == "clean"
    assert "49152" in b.validation_summary(size_only=True, target=target)
    assert b.coverage(None, [], "", {}) == {"kind": "sampling", "scope": ""}


def test_assemble_and_compiler_lines_map_back_to_the_candidate(tmp_path):
    b = CudaBackend()
    cand = 'extern "C" __global__ void k(float* y) {\n    y[0] = 1.0f\n}\n'  # missing ';' on line 2
    full, header = b.assemble(None, cand)
    path = tmp_path / "cand.cu"
    path.write_text(full)
    proc = subprocess.run([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-cubin", str(path), "-o",
                           str(tmp_path / "o.cubin")], capture_output=True, text=True)
    assert proc.returncode != 0
    msg = b.rewrite_compiler_lines(None, proc.stdout + proc.stderr, header)
    # nvcc reports the missing ';' at the next token, the '}' on candidate line 3.
    assert header == 2 and "cand.cu(3): error" in msg and "cand.cu(5)" not in msg


def test_artifact_builder_is_the_track_builder():
    b = CudaBackend()
    assert isinstance(b.artifact_builder(math="safe"), tf.CudaTrackBuilder)
    assert b.artifact_builder().extra_flags == ("--use_fast_math",)
    with pytest.raises(ValueError):
        b.artifact_builder(diagnostic_profile="nope")


def test_evaluator_refuses_an_uncompiled_entry_before_any_launch():
    """The launch block names an entry that the preprocessor removed: abi_error, no GPU touched."""
    src = '''#if 0
extern "C" __global__ void vanished(float* y) { y[0] = 0.0f; }
#endif
extern "C" __global__ void present(float* y) { y[0] = 1.0f; }
/* taic-launch
kernel vanished grid=1 threads=32
*/
'''
    rep = tf.CudaTrackEvaluator().evaluate(tf.EvaluationRequest(specs=[], cases=[], rtol=0.0, atol_rel=0.0, source=src))
    assert rep["status"] == "abi_error" and "vanished" in rep["detail"], rep


V1_DATA_PATH = {"prepare_case", "baseline_runners", "baseline_runner", "prepare_correctness", "prepare_bench_sets"}


def test_backend_protocol_methods_are_present():
    """Every method of the reference's Backend protocol (tcenv/backends/base.py) exists on the CUDA
    backend, except the v1 task-object data path, which the track evaluator replaces."""
    import os
    import re
    from pathlib import Path

    base = Path(os.environ.get("REFERENCE_ROOT", "/root/reference")) / "tcenv" / "backends" / "base.py"
    if not base.is_file():
        pytest.skip("reference checkout not mounted")
    text = base.read_text(encoding="utf-8")
    body = text[text.index("class Backend(Protocol)"):]
    names = set(re.findall(r"^    def (\w+)\(", body, flags=re.M))
    missing = sorted(n for n in names - V1_DATA_PATH if not hasattr(CudaBackend, n))
    assert missing == []
