"""The bench's tokenize workload (host only) on a small corpus: both arms
print their line, the arms count the same tokens, and the all-core batch
pass agrees with the single-core pass."""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tokenize_workload_small(monkeypatch):
    sys.path.insert(0, REPO)
    import bench
    monkeypatch.setattr(bench, "TOKENIZE_ITEMS", 4000)
    ours = bench.run_tokenize(bench.parse(["--workload", "tokenize", "--steps", "1", "--warmup", "0"]))
    assert ours["value"] > 0 and ours["tokens_per_step"] > 0
    assert ours["batch_all_cores"]["value"] > 0
    ref = bench.run_tokenize(bench.parse(["--workload", "tokenize", "--impl", "reference", "--steps", "1",
                                          "--warmup", "0"]))
    assert ref["impl"] == "reference"
    if "unavailable" not in ref:  # the reference's Tokenizer built here (oracle/_ref)
        assert ref["value"] > 0 and ours["reference"]["kind"] == "reference"
