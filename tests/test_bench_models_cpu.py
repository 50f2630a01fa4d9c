"""The benchmark workloads of bench_models build well-formed batches (CPU, reduced row counts)."""

import argparse

import numpy as np
import pytest
import torch


@pytest.mark.parametrize("name", ["mpnet", "modernvbert"])
def test_bench_workload_batches(name):
    from representax_b200 import bench_models as B
    from representax_b200.tasks._batch import leading_rows, slice_rows

    model, task, execution, policy, make_batch, rows, info = B.BUILDERS[name](
        argparse.Namespace(rows=4, dropout=0.1, fp8="block"), None)
    batch = make_batch(np.random.default_rng(0))
    assert rows == 4
    assert leading_rows(batch.query) == 4
    assert batch.positive_mask.shape[0] == 4
    assert leading_rows(slice_rows(batch.document, 0, 2)) == 2
    assert info["unit_rows"] in ("pairs", "triplets")
    if name == "modernvbert":
        assert policy.fp8_block_scaled and "MXFP8" in info["precision"]
    if name == "modernvbert":
        ids = batch.document.input_ids
        assert int((ids == model.config.image_token_id).sum(1)[0]) == model.config.image_sequence_length
        assert int(batch.query.input_ids.max()) < model.config.text.vocab_size
    else:
        assert batch.positive_mask.shape == (4, 8)
        assert torch.equal(batch.positive_mask[:, :4], torch.eye(4, dtype=torch.bool))
