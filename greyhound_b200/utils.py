import torch


def get_default_device() -> str:
    """``cuda:<current>`` when a GPU is present, else ``cpu`` (src/greyhound/utils.py:4-7)."""
    if torch.cuda.is_available():
        return f"cuda:{torch.cuda.current_device()}"
    return "cpu"
