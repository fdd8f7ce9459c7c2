"""bench.py on the CPU: the reference arm's JSON line (the driver's contract) on small workloads, on
the default (block) workload and under torchrun as the driver launches N > 1, and the rule that the
GPU arm imports the oracle only in its CPU-baseline leg (cpu_sample)."""
import ast
import json
import socket
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_one_contract_line():
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "rmsnorm",
                        "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "GB/s"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
    for key in ("metric", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling", "dtype",
                "config"):
        assert key in d


def test_oracle_only_in_the_cpu_baseline_leg():
    tree = ast.parse((ROOT / "bench.py").read_text())
    allowed = {"cpu_sample"}

    def imports_oracle(node):
        return any((isinstance(n, ast.ImportFrom) and (n.module or "").startswith("oracle")) or
                   (isinstance(n, ast.Import) and any(a.name.startswith("oracle") for a in n.names))
                   for n in ast.walk(node))

    assert not any(imports_oracle(n) for n in tree.body if not isinstance(n, (ast.FunctionDef, ast.ClassDef)))
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and imports_oracle(node):
            assert node.name in allowed, node.name


def test_reference_arm_default_is_the_block_workload():
    """The driver's call carries no --workload: the reference arm then samples the block (config 5)
    in the block's metric, on a bounded sample that the line names."""
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["value"] > 0 and d["n_gpus"] == 1
    assert d["config"]["layers"] == 28 and d["config"]["global_batch"] == 32 and d["config"]["seq_len"] == 1024
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["sample"]


def test_reference_arm_under_torchrun_prints_one_line():
    """Launched as the driver launches N > 1 (torchrun, one process per rank): rank 0 alone samples
    and prints; the other ranks exit 0 without work and without a process group."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    p = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
                        "--impl", "reference", "--workload", "rmsnorm", "--gpus", "2", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0


def test_reference_arm_linear_geglu_line():
    """The fused projection + GEGLU workload's reference arm: the reference torch path on a row
    sample, in the fused kernel's metric (TFLOP/s)."""
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "linear_geglu",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    d = json.loads([l for l in p.stdout.splitlines() if l.startswith("{")][-1])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
