"""blackhole_b200: the HEX fused-MoE layer of BlackHole-Harness, rebuilt for B200 (sm_100a).

    from blackhole_b200.hex_moe import HexTier, hex_moe        # drop-in for blackhole_runtime.hex_moe
    from blackhole_b200 import vllm_hex                       # the "blackhole-hex" vLLM plugin

The compute lives in libhexmoe.so (C ABI: include/hexmoe.h); importing
blackhole_b200.hex_moe loads it and fails if it is missing.
"""

__version__ = "0.1.0"
