"""CPU tests of the comparison rows (the reference report's TMA-vs-LSU row,
results/report.html:550-559, extended with copy, GEMM and NVLink rows)."""

import json

from cuda_micro_bench_b200 import compare


def _doc(vals):
    res = {}
    for (sec, key), v in vals.items():
        res.setdefault(sec, {})[key] = ({"value": None, "unit": "N/A"} if v is None
                                        else {"value": v, "unit": "x"})
    return {"device": "NVIDIA B200", "architecture": "10.0", "sm_count": 148, "results": res}


def test_rows_read_the_reports_keys_and_mark_the_best():
    doc = _doc({("memory_dram", "read_bw_gibps"): 6000.0, ("tma", "tma_g2s_load_bw_gibps"): 6020.0,
                  ("p2p", "ring_store_link_gbps"): 680.0, ("p2p", "ring_bulk_link_gbps"): 675.0,
                  ("p2p", "ring_copy_engine_link_gbps"): 745.0})
    rows = {name: (vals, best) for name, _, vals, best in compare.rows(doc)}
    vals, best = rows["DRAM read bandwidth"]
    assert [v for _, v in vals] == [6000.0, 6020.0] and best.startswith("TMA")
    vals, best = rows["NVLink ring, egress per GPU"]
    assert best == "copy engines"
    # rows whose keys the run did not log
    vals, best = rows["BF16 tensor throughput"]
    assert [v for _, v in vals] == [None, None, None, None] and best is None


def test_markdown_and_cli(tmp_path, capsys):
    doc = _doc({("memory_dram", "copy_bw_gbps"): 6500.0, ("tma", "tile_copy_bw_gbps"): 6100.0,
                  ("tensor_core_extended", "bf16_m16n8k16_throughput_TFs"): 488.0,
                  ("tensor_core_tcgen05", "bf16_gemm_8192_tflops"): 1519.0,
                  ("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_tflops"): None})
    md = compare.markdown(doc)
    assert "| DRAM copy bandwidth (read + write) | LSU copy stream (best) | 6,500.0 GB/s |  |" in md
    assert "3.11x" in md  # 1519 / 488
    assert "die-split order" in md and "plain tile order" in md
    assert "n/a" in md
    path = tmp_path / "r.json"
    path.write_text(json.dumps(doc))
    assert compare.main([str(path)]) == 0
    assert "NVLink all-to-all" in capsys.readouterr().out
