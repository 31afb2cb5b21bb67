"""Shared constants of the streaming semi-CRF (streaming/constants.py:10 of the reference)."""

NEG_INF = -1e9
