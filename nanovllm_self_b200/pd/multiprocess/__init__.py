"""Persistent prefill/decode worker processes, their control plane and the P/D pool driver."""
