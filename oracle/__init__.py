"""CPU oracle for the decode-attention path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this
package, and only as the checker or the timed CPU baseline. The product (kernel_optim_b200) never
imports it and has no CPU fallback.

Contents
* bf16.py       bf16 <-> fp32 bit helpers (round-to-nearest-even), numpy.
* prologue.py   restatement of the reference's QK-norm + RoPE + KV append
                (GodRishUniverse/kernel_optim engine/kernels/fused.py:54-96) with a fixed fp32
                summation order, and the Transformers Qwen3 modules it must agree with.
* attention.py  fp32 SDPA decode-attention oracle (the north-star tolerance target), and a numpy
                restatement of the reference's split-K kernel + LSE combine (fused.py:138-234).
* epilogue.py   restatement of the decode step's row kernels and projection epilogues (add +
                RMSNorm, SwiGLU, residual, LM-head argmax) in the reference's cast order.
* cpu_path.py   the reference's CPU path (Transformers' sdpa attention, repeat_kv and enable_gqa
                forms) used as the timed CPU baseline.

How the oracle is pinned: the reference's own tests hold no vectors for this path
(tests/test_client.py only mocks an HTTP client) and its Triton kernels need a GPU. The oracle is
therefore pinned against the reference's declared native path, which is what its judge replays
(QWEN_ENGINE_CONTRACT.md:105-123): Transformers' Qwen3RMSNorm / Qwen3RotaryEmbedding /
apply_rotary_pos_emb and torch's scaled_dot_product_attention, run on CPU in this container.
tests/golden/make_golden.py writes those outputs as committed fixtures.
"""
