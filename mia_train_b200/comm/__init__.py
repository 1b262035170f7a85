"""Peer-memory communication over NVLink: CUDA-IPC buffers (`ipc`) and the workspace of the fused
tensor-parallel collective GEMMs (`tp_workspace`)."""
