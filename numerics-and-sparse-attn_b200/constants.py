"""Workload constants, same names and values as the reference's constants.py:6-19."""

BATCH = 32
N_HEADS = 64
N_KV_HEADS = 8
GQA_GROUP = N_HEADS // N_KV_HEADS
D_HEAD = 128
BLOCK_N = 128

SINK_SIZE = 4          # StreamingLLM attention-sink size
RESIDUAL_SIZE = 128    # KIVI: most recent tokens kept in fp16
GROUP_SIZE = 32        # KIVI quantization group size (K and V)
QUANT_BITS = 2         # KIVI main-cache precision

CONTEXT_LENGTHS = [8_192, 16_384, 32_768, 65_536, 131_072, 163_840]
WINDOW_SIZES = [0, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384]
