"""greyhound_b200: B200-native (sm_100a) drop-in for greyhound's chunked linear
cross-entropy hot path (``nn.functional`` / ``ops`` / ``kernels`` layers)."""

VERSION = "0.1.0"
VERSION_SHORT = "0.1"
