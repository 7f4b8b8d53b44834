"""The "blackhole-hex" vLLM quantization method on this build's sm_100a layer.

Drop-in for the reference plugin (runtime/blackhole_runtime/vllm_hex.py): the
same quantization name, the same checkpoint tensor names
(<experts prefix>.tier<L>.experts and .tier<L>.<proj>.<part>, vllm_hex.py:32)
and the same vLLM hooks, with the routed experts running through
blackhole_b200.hex_moe.  A folder written for the reference serves unchanged:

    vllm serve <blackhole-hex folder>

once register() has run in the vLLM process (the general-plugin entry point
`blackhole_b200.vllm_hex:register`, declared in pyproject.toml).

Differences from the reference, each deliberate:
  * minimum capability 100: the kernels are built for sm_100a only;
  * the layer's C-ABI handle (and its tiled index copy) is built in
    process_weights_after_loading, before vLLM captures CUDA graphs;
  * topk ids reach the kernels in the dtype vLLM produces (int32 or int64;
    no copy to int64 as at vllm_hex.py:146);
  * the model-specific n-gram embedding patch (vllm_hex.py:41-64) is left out:
    the vLLM here has no such model.
Tensor and expert parallelism stay refused (vllm_hex.py:101-102); multi-GPU
runs use blackhole_b200.ep outside vLLM.
"""

from __future__ import annotations

import re

import torch

NAME = "blackhole-hex"
HEAD_FILL = -1.0e4   # logit of a token an output-trimmed LM head cannot write (vllm_hex.py:29-30)
PARTS = ("idx", "block_scale", "expert_scale", "levels")
PROJS = ("gate_proj", "up_proj", "down_proj")
# expert-relative names: tier<L>.experts, tier<L>.<proj>.<part>
_TENSOR = re.compile(r"^(?:.*\.)?tier(?P<L>\d+)\.(?:(?P<ids>experts)|(?P<proj>gate_proj|up_proj|down_proj)\."
                     r"(?P<part>idx|block_scale|expert_scale|levels))$")


def param_name(name: str) -> str | None:
    """The layer parameter a checkpoint tensor loads into (None: not a HEX tensor)."""
    m = _TENSOR.match(name)
    if not m:
        return None
    return f"hex_t{m['L']}_experts" if m["ids"] else f"hex_t{m['L']}_{m['proj']}_{m['part']}"


def build_tiers(layer: torch.nn.Module, num_experts: int, inter: int, hidden: int) -> list:
    """The prepared HexTier list from a layer's loaded hex_t* parameters, the
    16-level tier first; ValueError when a tier is incomplete, its shapes do not
    match the model, or an expert has no weights (vllm_hex.py:123-140)."""
    from blackhole_b200.hex_moe import HexTier
    name = getattr(layer, "layer_name", type(layer).__name__)
    params = dict(layer.named_parameters(recurse=False))
    levels = sorted({int(n.split("_")[1][1:]) for n in params if n.startswith("hex_t")}, reverse=True)
    if not levels:
        raise ValueError(f"{NAME}: no HEX experts were loaded for {name}")
    tiers, held = [], torch.zeros(num_experts, dtype=torch.bool)
    for L in levels:
        if L not in (8, 16):
            raise ValueError(f"{NAME}: {name} tier{L}: HEX tables have 8 or 16 levels")
        try:
            ids = params[f"hex_t{L}_experts"].data
            proj = [{p: params[f"hex_t{L}_{j}_{p}"].data for p in PARTS} for j in PROJS]
        except KeyError as e:
            raise ValueError(f"{NAME}: {name} tier{L} is missing {e.args[0]}") from None
        tier = HexTier(L.bit_length() - 1, ids, *proj).prepare(num_experts)
        if tier.dims() != (inter, hidden):
            raise ValueError(f"{NAME}: {name} tier{L} is [I, H] = {tier.dims()}, the model has {(inter, hidden)}")
        held[ids.long().cpu()] = True
        tiers.append(tier)
    if not bool(held.all()):
        missing = (~held).nonzero().flatten().tolist()
        raise ValueError(f"{NAME}: {name} has no weights for experts {missing[:8]}")
    return tiers


def register() -> None:
    """vLLM general-plugin entry point: registers the quantization method.
    Safe to call more than once."""
    if _registered:
        return
    from vllm.model_executor.layers.quantization import register_quantization_config
    from vllm.model_executor.layers.fused_moe import FusedMoEMethodBase, RoutedExperts
    from vllm.model_executor.layers.linear import LinearBase, UnquantizedLinearMethod
    from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
    from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead, UnquantizedEmbeddingMethod

    class HexHeadMethod(UnquantizedEmbeddingMethod):
        """Output-trimmed LM head: only the kept vocabulary rows are multiplied.

        The reference computes every logit and then adds a -1e4 mask outside the
        kept ids (vllm_hex.py:78-93).  Here the kept rows of the weight are
        gathered once after loading into a [K, hidden] matrix; apply() runs that
        K-row GEMM and scatters its columns into logits pre-filled with HEAD_FILL,
        so the head reads and multiplies K of the V rows.  Kept logits are the
        same GEMM values; a dropped token's logit is HEAD_FILL itself (the
        reference's is its true logit - 1e4): either way it is never sampled."""

        def __init__(self, ids):
            super().__init__()
            self.keep = sorted({int(i) for i in ids})

        def process_weights_after_loading(self, layer) -> None:
            super().process_weights_after_loading(layer)
            w = layer.weight
            keep = torch.as_tensor(self.keep, dtype=torch.long, device=w.device)
            if keep.numel() and (int(keep.min()) < 0 or int(keep.max()) >= w.shape[0]):
                raise ValueError(f"{NAME}: head_ids outside the vocabulary of {w.shape[0]} rows")
            layer.register_buffer("hex_head_keep", keep, persistent=False)
            layer.register_buffer("hex_head_rows", w.index_select(0, keep).contiguous(), persistent=False)

        def apply(self, layer, x, bias=None):
            kept = torch.nn.functional.linear(x, layer.hex_head_rows,
                                              None if bias is None else bias.index_select(0, layer.hex_head_keep))
            out = torch.full((*x.shape[:-1], layer.weight.shape[0]), HEAD_FILL, dtype=kept.dtype, device=x.device)
            out.index_copy_(-1, layer.hex_head_keep, kept)
            return out

    class HexMoEMethod(FusedMoEMethodBase):
        """Routed experts of one MoE layer as HEX tiers on the sm_100a layer."""

        def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                           **extra_weight_attrs):
            if getattr(self.moe, "tp_size", 1) != 1 or getattr(self.moe, "ep_size", 1) != 1:
                raise ValueError(f"{NAME} runs each MoE layer on one GPU: --tensor-parallel-size 1, no expert parallel")
            layer.hex_shape = (num_experts, hidden_size, intermediate_size_per_partition)
            layer.hex_tiers = []
            # tier shapes are known only from the checkpoint: parameters are made as they load
            layer.load_weights = lambda weights: self.load(layer, weights)

        def load(self, layer, weights):
            for name, t in weights:
                key = param_name(name)
                if key is None:
                    raise ValueError(f"{NAME}: unexpected expert tensor {getattr(layer, 'layer_name', '')}.{name} "
                                     "(expected tier<L>.<proj>.<part> and tier<L>.experts)")
                dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else t.device
                layer.register_parameter(key, torch.nn.Parameter(t.to(dev), requires_grad=False))
                yield key

        def process_weights_after_loading(self, layer) -> None:
            E, H, I = layer.hex_shape
            layer.hex_tiers = build_tiers(layer, E, I, H)
            if layer.hex_tiers[0].gate_proj["idx"].is_cuda:
                from blackhole_b200.hex_moe import layer_for
                layer_for(layer.hex_tiers)    # the C-ABI layer (tiled index copy) before graph capture

        def get_fused_moe_quant_config(self, layer):
            return None

        def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
            from blackhole_b200.hex_moe import hex_moe
            return hex_moe(x, topk_weights, topk_ids, layer.hex_tiers)

    @register_quantization_config(NAME)
    class HexConfig(QuantizationConfig):
        def __init__(self, cfg: dict):
            super().__init__()
            self.cfg = dict(cfg)
            self.head_ids = self.cfg.get("head_ids")

        def get_name(self):
            return NAME

        def get_supported_act_dtypes(self):
            return [torch.bfloat16, torch.float16]

        @classmethod
        def get_min_capability(cls) -> int:
            return 100

        @staticmethod
        def get_config_filenames():
            return []

        @classmethod
        def from_config(cls, config: dict):
            return cls(config)

        def get_quant_method(self, layer, prefix: str):
            if isinstance(layer, RoutedExperts):
                return HexMoEMethod(layer.moe_config)
            if isinstance(layer, ParallelLMHead) and self.head_ids:
                return HexHeadMethod(self.head_ids)
            if isinstance(layer, LinearBase):
                return UnquantizedLinearMethod()
            return None

    _registered.update(config=HexConfig, moe=HexMoEMethod, head=HexHeadMethod)


_registered: dict = {}   # the classes register() made (empty until it runs)
