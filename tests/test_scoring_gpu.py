"""The scoring forward (noise_b200.population.evaluate) against utils/eval.py:35-53's arithmetic.

The reference scores validation rows in batches of 16 under bf16 autocast, sums each batch's
per-token cross-entropy (loss_reduction='sum') into a float64 total and divides by the number of
predictions. Here the same mean comes from the sigma = 0 population forward, batch by batch, summed in
float64. Compared with the float32 CPU oracle of GPT.forward (itself pinned to the reference's
GPT.forward by tests/golden/forward.npz) on 18 synthetic rows of 2049 tokens: one full batch of 16 and a
ragged one of 2. Tolerance: relative 1e-4 on the mean (bf16 GEMM operands against float32).
"""
import pytest
import torch

from noise_b200.data import zipf_tokens

pytestmark = pytest.mark.gpu


def test_evaluate_matches_reference_arithmetic():
    from noise_b200.model import Weights
    from noise_b200.population import evaluate
    from oracle import model as om
    rows = zipf_tokens(18, 2049, seed=13)
    w = Weights('cuda', seed=0)
    got = evaluate(w, rows, batch=16)
    p = om.make_params(0)
    total, count = 0.0, 0
    with torch.no_grad():
        for batch in rows.split(16):  # the reference's batching and float64 sum
            total += float(om.forward(p, batch[:, :-1], batch[:, 1:], reduction='sum').double())
            count += batch[:, 1:].numel()
    want = total / count
    print('evaluate', got, 'oracle', want, 'rel', abs(got - want) / want)
    assert abs(got - want) / want <= 1e-4
