"""Benchmark record files: ResultLog prints each record and appends it, with metadata, to a
JSON-lines file; disabled instances (ranks other than 0) stay silent."""
import json

from originccl_b200.utils.results import ResultLog


def test_records_are_printed_and_appended(tmp_path, capsys):
    path = tmp_path / "bench" / "results" / "sweep.jsonl"
    with ResultLog("sweep", str(path)) as log:
        log({"op": "allreduce", "bytes": 8, "busbw_gbs": 1.5})
        log(json.dumps({"op": "allreduce", "bytes": 16, "busbw_gbs": 2.5}))
    with ResultLog("sweep", str(path)) as log:  # a second run appends
        log({"op": "allreduce", "bytes": 32})
    printed = [json.loads(x) for x in capsys.readouterr().out.splitlines()]
    assert [r["bytes"] for r in printed] == [8, 16, 32]
    recs = [json.loads(x) for x in path.read_text().splitlines()]
    assert [r["bytes"] for r in recs] == [8, 16, 32]
    assert all(r["bench"] == "sweep" and r["utc"].endswith("Z") and r["host"] for r in recs)


def test_disabled_log_is_silent(tmp_path, capsys):
    path = tmp_path / "r.jsonl"
    log = ResultLog("dp_bench", str(path), enabled=False)
    log({"x": 1})
    log.close()
    assert capsys.readouterr().out == "" and not path.exists()
