"""mdlc_b200 — B200-native (sm_100a) execution backend for mdlc's Graph IR."""

__version__ = "0.1.0"
