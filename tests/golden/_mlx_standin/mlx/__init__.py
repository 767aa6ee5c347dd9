"""NumPy stand-in for the few ``mlx`` names the reference's KV quantizer uses.

Used only by ``tests/golden/gen_golden.py`` to execute the reference's own
``quantize_tensor`` / ``dequantize_tensor`` source when generating golden
vectors (MLX itself is not installable here).  Element-wise ops on bf16/fp16
arrays are evaluated as "float32 op, then round to the array dtype".
"""
