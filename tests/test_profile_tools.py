"""Host-side measurement tooling: the ncu raw-CSV traffic reader that fills the traffic table bench.py reads."""

import json

from smolvla_mujoco_libero_b200 import profile


def _csv(tmp_path, unit="Mbyte"):
    p = tmp_path / "raw.csv"
    p.write_text(
        '"ID","Kernel Name","dram__bytes_read.sum","dram__bytes_write.sum"\n'
        f'"","","{unit}","{unit}"\n'
        '"0","flow_kernel(svla::FlowArgs)","1,000.5","24.5"\n'
        '"1","gemm_sm100_kernel<0, 256>","10","10"\n'
        '"2","flow_kernel(svla::FlowArgs)","999.5","23.5"\n')
    return p


def test_ncu_traffic_mean_per_launch_with_units(tmp_path):
    b, n = profile.ncu_traffic(str(_csv(tmp_path)), "flow_kernel")
    assert n == 2 and abs(b - 1024.0e6) < 1.0
    b, n = profile.ncu_traffic(str(_csv(tmp_path, "Kbyte")), "gemm_sm100")
    assert n == 1 and abs(b - 20.0e3) < 1e-6


def test_update_traffic_scales_and_keeps_other_entries(tmp_path):
    table = tmp_path / "traffic.json"
    table.write_text(json.dumps({"other": {"dram_bytes_per_launch": 5.0}}))
    e = profile.update_traffic(str(table), "flow_kernel_b1", str(_csv(tmp_path)), "flow_kernel", 4.0, "small case")
    assert abs(e["dram_bytes_per_launch"] - 4 * 1024.0e6) < 4.0 and e["launches"] == 2
    t = json.loads(table.read_text())
    assert set(t) == {"other", "flow_kernel_b1"} and t["flow_kernel_b1"]["note"] == "small case"
