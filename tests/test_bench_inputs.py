"""bench.py generates the C4 headline inputs itself (numpy restatement of
the benchmark's splitmix64 / Box-Muller streams, no oracle import); they must
be the same bytes as the CPU oracle's generator gives for configuration C4, so
the GPU arm and the CPU baseline compute on identical data."""
import os
import sys

import numpy as np
import torch

import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
import bench  # noqa: E402


def test_seeded_c4_inputs_equal_the_oracle_generator():
    m, k, n = 96, 1536, 6144
    x, blob_dev, bias, blob_host, bias_host = bench.seeded_c4_inputs(torch, torch.device("cpu"), m, k, n)
    c = O.make_w8a8(3, "C4", m, k, n, 0.005, True, 1)
    np.testing.assert_array_equal(x.numpy().view(np.uint32), c.x.view(np.uint32))
    np.testing.assert_array_equal(bias_host.view(np.uint32), c.bias.view(np.uint32))
    # the blobs differ only in the header's signature field: compare weights, scales, sums, inverse
    np.testing.assert_array_equal(blob_host[128:], c.blob[128:])
    np.testing.assert_array_equal(O.w8a8_unpack(blob_host, k, n), c.w)


def test_seeded_normal_without_outliers_matches():
    a = bench.seeded_normal(1001, 0.02, 0.0, 1.0, bench.tensor_seed(1, 2))
    b = O.normal(1001, 0.02, 0.0, 1.0, O.tensor_seed(1, 2))
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
