"""The run records kept in the reference's own file formats (committed files; no GPU needed).

- kernel-rsi_b200/hardware/nvidia_b200.json, written on a B200 by tests/make_hardware_record.py in
  the layout of the reference's hardware/<device>.json (tools/hw.py:90-183).  The reference's tools
  read `device`, `tflops` fp16 / bf16 / fp32 / tf32 and the larger of `bw_copy_gbs` and
  `bw_read_gbs` (tools/common.py:35-64), from the file named by the device's slug.
- kernel-rsi_b200/library/replay/nvidia_b200.json, written by tests/make_replay_record.py in the
  layout of library/replay/<gpu>.json (tools/replay.py:24-59).
"""
import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests"))

import make_hardware_record as hw  # noqa: E402

HW_RECORD = ROOT / "kernel-rsi_b200" / "hardware" / "nvidia_b200.json"
REPLAY_RECORD = ROOT / "kernel-rsi_b200" / "library" / "replay" / "nvidia_b200.json"

# Keys of the reference's hardware record (its H20 file), less the Triton launch probe this build
# replaces with launch_us_krsi.
HW_KEYS = {"device", "sm", "sms", "l2_mb", "memory_gb", "tflops", "bw_copy_gbs", "bw_read_gbs", "bw_write_gbs",
           "ridge_flop_per_byte", "default_half_dtype", "features", "smem_per_block_kb", "regs_per_sm",
           "sm_clock_mhz", "triton", "launch_us_torch", "launch_us_graph_replay", "ncu", "torch"}
HW_FEATURES = {"bf16_tensor_cores", "tf32", "fp8", "hopper_wgmma_tma"}


def test_device_slug_gives_the_reference_file_names():
    assert hw.device_slug("NVIDIA H20-3e") == "nvidia_h20_3e"   # hardware/nvidia_h20_3e.json
    assert hw.device_slug("NVIDIA B200") == "nvidia_b200"
    assert hw.device_slug("  NVIDIA GeForce RTX 4090 ") == "nvidia_geforce_rtx_4090"


def test_ridge_reproduces_the_reference_h20_record():
    # tflops and bandwidths of the reference's hardware/nvidia_h20_3e.json and its ridge figures
    tflops = {"fp16": 141.0, "bf16": 138.6, "fp32": 25.8, "tf32": 69.7, "fp8": 278.7,
              "skinny_bf16": {"M16xN4096xK4096": 12.2}}
    assert hw.ridge(tflops, max(2247, 2610)) == {"fp16": 54.0, "bf16": 53.1, "fp32": 9.9, "tf32": 26.7,
                                                 "fp8": 106.8}


def test_hardware_record_has_the_reference_layout():
    rec = json.loads(HW_RECORD.read_text())
    assert HW_RECORD.stem == hw.device_slug(rec["device"])
    assert HW_KEYS <= set(rec), sorted(HW_KEYS - set(rec))
    assert HW_FEATURES <= set(rec["features"])
    tf = rec["tflops"]
    for k in ("fp16", "bf16", "fp32", "tf32", "fp8"):
        assert isinstance(tf[k], (int, float)) and tf[k] > 0, k
    assert set(tf["skinny_bf16"]) == {f"M{m}xN4096xK4096" for m in (16, 64, 256, 1024)}
    for k in ("bw_copy_gbs", "bw_read_gbs", "bw_write_gbs"):
        assert isinstance(rec[k], int) and rec[k] > 0, k
    assert rec["ridge_flop_per_byte"] == hw.ridge(tf, max(rec["bw_copy_gbs"], rec["bw_read_gbs"]))
    assert rec["default_half_dtype"] == "bf16" and rec["sm"] == "sm_100" and rec["sms"] == 148


def test_hardware_record_gives_the_reference_peaks():
    """tools/common.py:55-64 (peaks): bf16 work divides by tflops.bf16 and max(copy, read)."""
    rec = json.loads(HW_RECORD.read_text())
    flops = rec["tflops"]["bf16"] * 1e12
    bw = max(rec["bw_copy_gbs"], rec["bw_read_gbs"]) * 1e9
    # a measured B200: dense bf16 between 1 and 2.25 PFLOP/s, HBM between 5 and 8 TB/s
    assert 1.0e15 < flops < 2.25e15
    assert 5.0e12 < bw < 8.0e12


REPLAY_OP_KEYS = {"pass", "device", "torch", "cuda", "triton", "reference_us", "kernel_us", "speedup",
                  "significance", "compiled"}
REPLAY_COMPILED_KEYS = {"pass", "kernel_us", "reference_us", "speedup", "significance"}


@pytest.mark.parametrize("op", ["rmsnorm", "geglu", "relpos_attention", "linear_geglu", "t5_bias"])
def test_replay_record_has_the_reference_layout(op):
    rec = json.loads(REPLAY_RECORD.read_text())
    assert {"versions", "library", "regions"} <= set(rec)
    assert set(rec["versions"]) == {"device", "torch", "cuda", "triton"}
    entry = rec["library"][op]
    assert set(entry) == REPLAY_OP_KEYS
    assert set(entry["compiled"]) == REPLAY_COMPILED_KEYS
    assert entry["pass"] and entry["compiled"]["pass"]
    assert entry["device"] == rec["versions"]["device"] == "NVIDIA B200"
    assert entry["significance"] in ("faster", "slower", "within noise")   # tools/common.py:467-473
