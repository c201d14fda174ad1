"""Chunked overlap of the TP sequence all-gather / reduce-scatter with GEMM.

Column-parallel: the sequence dimension is gathered chunk by chunk; the GEMM
on chunk ``i`` runs on the compute stream while chunk ``i+1`` is in flight on
the communication stream.  Row-parallel: the GEMM output is produced per
destination chunk and each chunk's reduce-scatter starts as soon as it is
ready.
"""
ENABLED = False
