"""The reference benchmark's CSV row from the GPU path."""

import csv

import pytest
import torch

from streaming_attention_b200 import bench_csv

pytestmark = pytest.mark.gpu


def test_one_row_matches_the_reference_state_accounting(tmp_path):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    out = tmp_path / "r.csv"
    rows = bench_csv.main(["--sweep-n", "64", "--d", "16", "--dv", "16", "--block-size", "64", "--repeats", "1",
                           "--out", str(out)])
    r = rows[0]
    # the reference's own sample row for these arguments (benchmark_sample.csv, first row)
    assert (r["article_final_state_bytes"], r["article_max_state_bytes"], r["article_max_coreset_items"]) == \
        (14628, 18468, 63)
    assert r["classical_kv_bytes"] == 8192 and r["classical_naive_scores_bytes"] == 16384
    assert r["rel_l2"] < 1e-2
    with open(out) as f:
        back = list(csv.DictReader(f))
    assert list(back[0].keys()) == bench_csv.COLUMNS and int(back[0]["n"]) == 64
