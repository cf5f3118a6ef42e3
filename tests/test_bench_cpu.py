"""Host-side pieces of bench.py: the DRAM-traffic record is used only for the sources and
workload it was captured on, and the headline workload string names the metric's 32K case."""
import json

import bench


def test_headline_workload_is_the_32k_case():
    wl = bench._workload(bench.HEAD)
    assert "S=32768" in wl and "B=8" in wl and "Hq=28" in wl and "Hk=4" in wl and "R=128" in wl
    assert bench.CFG1["S"] == 16384


def test_traffic_record_matches_current_sources():
    with open(bench.TRAFFIC_FILE) as f:
        rec = json.load(f)
    assert rec["source_sha256"] == bench._sources_sha(), "profiles traffic record is stale: recapture it"
    assert rec["workload"] == bench._workload(bench.HEAD)
    assert bench._measured_traffic(bench._workload(bench.HEAD)) == rec["dram_bytes_per_launch"]
    assert rec["dram_bytes_per_launch"] == rec["dram_bytes_read"] + rec["dram_bytes_write"]


def test_traffic_record_ignored_for_other_workloads_and_sources(tmp_path, monkeypatch):
    assert bench._measured_traffic(bench._workload(bench.CFG1)) is None
    with open(bench.TRAFFIC_FILE) as f:
        rec = json.load(f)
    rec["source_sha256"] = "0" * 64
    stale = tmp_path / "traffic.json"
    stale.write_text(json.dumps(rec))
    monkeypatch.setattr(bench, "TRAFFIC_FILE", str(stale))
    assert bench._measured_traffic(bench._workload(bench.HEAD)) is None
