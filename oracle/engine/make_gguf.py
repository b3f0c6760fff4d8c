"""Writes the synthetic Qwen3-0.6B-architecture GGUF of the config-2 check
(test infrastructure): random-init bf16 weights from a seed, in the tensor
names and metadata keys the Genllm Qwen3 loader reads
(src/model/Qwen3.cpp:23-45 keys; :64-199 tensors; tied LM head, :94), norm
weights in f32 (the engine's RMSNorm reads them so,
src/backend/cpu/normalization.cpp:147). Matrices are N(0, 1/fan_in) so that
activations stay O(1) through the layers; the embedding (and tied LM head)
is N(0, 1), which spreads the logits so that greedy picks have margins well
above bf16 rounding. The two projections that write the residual stream
(attn_output, ffn_down) get a gain of OUT_GAIN, so that the stream is
dominated by what the layers compute from the context rather than by the
input token's own embedding (with a tied head that would make greedy decode
repeat the last token).

    python make_gguf.py OUT [--layers 28] [--vocab 151936] [--seed 1]
"""
import argparse

import numpy as np


OUT_GAIN = 4.0


def bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("out")
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--hidden", type=int, default=1024)
    ap.add_argument("--ffn", type=int, default=3072)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--seed", type=int, default=1)
    a = ap.parse_args()
    import gguf

    D = 128
    rng = np.random.default_rng(a.seed)
    w = gguf.GGUFWriter(a.out, "qwen3")
    w.add_uint32("qwen3.embedding_length", a.hidden)
    w.add_uint32("qwen3.block_count", a.layers)
    w.add_uint32("qwen3.attention.head_count", a.heads)
    w.add_uint32("qwen3.attention.head_count_kv", a.kv_heads)
    w.add_uint32("qwen3.attention.key_length", D)
    w.add_uint32("qwen3.attention.value_length", D)
    w.add_uint32("qwen3.feed_forward_length", a.ffn)
    w.add_float32("qwen3.attention.layer_norm_rms_epsilon", 1e-6)
    w.add_float32("qwen3.rope.freq_base", 1e6)
    w.add_uint32("qwen3.context_length", 4096)
    # The loader takes the vocabulary size from the tokenizer's token list
    # (src/model/Qwen3.cpp:35-38); placeholder strings (ids are fed directly).
    w.add_array("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(a.vocab)])

    def mat(rows, cols, gain=1.0):
        return bf16(rng.standard_normal((rows, cols), dtype=np.float32) * (gain / np.sqrt(cols)))

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    BF16 = gguf.GGMLQuantizationType.BF16
    w.add_tensor("token_embd.weight", bf16(rng.standard_normal((a.vocab, a.hidden), dtype=np.float32)), raw_dtype=BF16)
    w.add_tensor("output_norm.weight", norm(a.hidden))
    for l in range(a.layers):
        p = f"blk.{l}"
        w.add_tensor(f"{p}.attn_norm.weight", norm(a.hidden))
        w.add_tensor(f"{p}.attn_q.weight", mat(a.heads * D, a.hidden), raw_dtype=BF16)
        w.add_tensor(f"{p}.attn_k.weight", mat(a.kv_heads * D, a.hidden), raw_dtype=BF16)
        w.add_tensor(f"{p}.attn_v.weight", mat(a.kv_heads * D, a.hidden), raw_dtype=BF16)
        w.add_tensor(f"{p}.attn_q_norm.weight", norm(D))
        w.add_tensor(f"{p}.attn_k_norm.weight", norm(D))
        w.add_tensor(f"{p}.attn_output.weight", mat(a.hidden, a.heads * D, OUT_GAIN), raw_dtype=BF16)
        w.add_tensor(f"{p}.ffn_norm.weight", norm(a.hidden))
        w.add_tensor(f"{p}.ffn_gate.weight", mat(a.ffn, a.hidden), raw_dtype=BF16)
        w.add_tensor(f"{p}.ffn_up.weight", mat(a.ffn, a.hidden), raw_dtype=BF16)
        w.add_tensor(f"{p}.ffn_down.weight", mat(a.hidden, a.ffn, OUT_GAIN), raw_dtype=BF16)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


if __name__ == "__main__":
    main()
