"""Test marks: the reference's `has_cuda` / `GPU_MARKS` / `requires_gpu`
(src/greyhound/testing.py:1-11) kept as they are there, because the
reference-style tests are written against exactly these names and marks."""

import pytest
import torch

has_cuda = torch.cuda.is_available()
GPU_MARKS = (pytest.mark.gpu, pytest.mark.skipif(not has_cuda, reason="Requires a GPU"))


def requires_gpu(func):
    for mark in GPU_MARKS:
        func = mark(func)
    return func
