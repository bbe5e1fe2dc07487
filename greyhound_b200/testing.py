"""Test marks, as in src/greyhound/testing.py:4-11."""

import pytest
import torch

has_cuda = torch.cuda.is_available()
GPU_MARKS = (pytest.mark.gpu, pytest.mark.skipif(not has_cuda, reason="Requires a GPU"))


def requires_gpu(func):
    for mark in GPU_MARKS:
        func = mark(func)
    return func
