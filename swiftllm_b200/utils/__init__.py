"""Logging, NVTX ranges, device timers and roofline helpers."""
