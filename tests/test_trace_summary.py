"""Trace summaries: interval unions, categories, comm/compute overlap, ncu CSV parsing (CPU)."""
import json

from flare_b200.utils.trace_summary import (categorize, interval_union, load_chrome_trace, summarize_events,
                                            summarize_ncu_csv)


def test_union_and_overlap(tmp_path):
    assert interval_union([(0, 2), (1, 3), (5, 6)]) == 4
    assert categorize("gemm_dist_tcgen05_kernel") == "fused_collective"
    assert categorize("ncclDevKernel_AllReduce") == "nccl"
    assert categorize("attn_fwd_kernel") == "attention" and categorize("gemm_tcgen05_kernel") == "gemm"
    ev = [{"ph": "X", "cat": "kernel", "name": "gemm_tcgen05_kernel", "ts": 0, "dur": 10, "tid": 7},
          {"ph": "X", "cat": "kernel", "name": "ncclDevKernel_AllReduce", "ts": 5, "dur": 10, "tid": 9},
          {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "ts": 0, "dur": 100}]
    p = tmp_path / "t.json"
    p.write_text(json.dumps({"traceEvents": ev}))
    s = summarize_events(load_chrome_trace(str(p)))
    assert s["span_us"] == 15 and s["busy_us"] == 15
    assert s["comm_overlapped_us"] == 5 and s["comm_exposed_us"] == 5
    assert s["categories"]["gemm"]["count"] == 1


def test_ncu_csv(tmp_path):
    rows = ['"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"',
            '"0","emb_fwd_kernel","gpu__time_duration.sum","usecond","100"',
            '"1","gemm_tcgen05_kernel","gpu__time_duration.sum","nsecond","300,000"',
            '"2","emb_fwd_kernel","gpu__time_duration.sum","usecond","100"']
    p = tmp_path / "l.csv"
    p.write_text("==PROF== noise\n" + "\n".join(rows) + "\n")
    s = summarize_ncu_csv(str(p))
    assert s["total_us"] == 500 and s["kernels"][0]["kernel"] == "gemm_tcgen05_kernel"
    assert s["kernels"][1]["launches"] == 2 and abs(s["categories"]["fused_collective"]["share"] - 0.4) < 1e-9
