from greyhound_b200.nn import functional

__all__ = ["functional"]
