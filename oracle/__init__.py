"""ORACLE — test infrastructure only.

A CPU restatement of the reference's ONNX Runtime CPU path (interp.py), an independent ONNX
decoder (onnx_decode.py) and a plain-C cross-check (ref_small.c).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import anything here; the product
library never does.
"""
