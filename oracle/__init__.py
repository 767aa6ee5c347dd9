"""CPU oracle for the quantized-weight / quantized-KV hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker (never as the thing measured for the GPU path).

Modules
-------
``fp``        float helpers: round-to-nearest-even into bf16 / fp16.
``affine``    MLX affine group quantization (weights): quantize, dequantize,
              quantized_matmul, gather_qmm.  Restated from the format contract
              (group 64, scale=(max-min)/(2^bits-1), bias=min, LSB-first
              uint32 packing; unpack order as in
              ``mlx_flash_compress/mixed_precision.py:150-171``).
``kv_sym``    the reference's own symmetric KV quantizer restated op by op
              (``mlx_flash_compress/quantized_kv_cache.py:68-234``).
``attn``      GQA decode attention over dequantized K/V (the consumer of
              ``quantized_kv_cache.py:311-358``).
``moe``       router softmax/top-k/renorm and the routed SwiGLU expert MLP
              (``mlx_flash_compress/expert_streaming.py:224-241, 439-472``).
``decoder``   one decode step of a Qwen3-MoE-shaped decoder built from the
              pieces above.
``q4_0_gemv.c`` the Metal ``flash_dequant_gemv_q4`` shader math
              (``mlx_flash_compress/kernels/flash_dequant.metal:19-49``) as C.

Parity status: the KV quantizer is pinned by executing the reference's own
``quantize_tensor``/``dequantize_tensor`` source (with a NumPy stand-in for
``mlx.core``, see ``tests/golden/gen_golden.py``).  The affine weight format
is pinned for unpack order and dequantization by the reference's own
``mixed_precision.requantize_4bit_to_2bit``; the quantizer's scale/bias rule
itself lives inside MLX (absent here) and is therefore "parity unpinned"
against real MLX.
"""
