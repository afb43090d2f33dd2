"""Model-level mirror: TESMConfig, FeedForward, MixerModel, TESMLMHeadModel.

Same field names, defaults (except ``kernel_backend``, which defaults to
``"b200"``), constructor signatures, state_dict keys and seeded-init order as
the reference (WANGLILIN360/tesm):
  TESMConfig        tesm_ssm/models/config_tesm.py:19-480
  FeedForward       tesm_ssm/models/mixer_seq_simple.py:25-67
  MixerModel        tesm_ssm/models/mixer_seq_simple.py:70-242
  TESMLMHeadModel   tesm_ssm/models/mixer_seq_simple.py:245-345, generate :617-703
  _init_weights     tesm_ssm/models/mixer_seq_simple.py:790-803
The training presets of TESMConfig and the vocabulary-suppression / semantic
activation logits paths are outside the inference hot path and are not mirrored
(their buffers are, so checkpoints load strictly).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from functools import partial
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from . import layers
from .modules import BitLinear, Block, RMSNorm, TESM_SISO, TESMMIMO_Optimized


@dataclass
class TESMConfig:
    d_model: int = 768
    n_layer: int = 24
    d_intermediate: int = 2048
    vocab_size: int = 151936
    max_seq_len: int = 2048
    pad_token_id: int = 0
    eos_token_id: Optional[int] = None
    label_ignore_index: int = -100
    gradient_checkpointing: bool = False
    tie_embeddings: bool = True
    dropout: float = 0.0
    rms_norm: bool = True
    residual_in_fp32: bool = True
    norm_epsilon: float = 1e-5
    initializer_range: float = 0.02
    rescale_prenorm_residual: bool = True
    bit_eps: float = 1e-5
    bit_threshold: float = 0.5
    vocab_suppression: bool = False
    suppression_bias: float = -10.0
    semantic_activation: bool = True
    semantic_activation_strength: float = 0.5
    semantic_activation_threshold: float = 0.1
    use_mimo: bool = False
    n_heads: int = 4
    d_state: int = 256
    expand: int = 2
    ent_rank: int = 64
    entanglement_scale: float = 0.2
    entanglement_threshold: float = 0.1
    entanglement_init: float = 0.3
    entanglement_window: int = 16
    entanglement_block_size: int = 256
    state_scan_chunk_size: int = 16
    use_triton_kernels: bool = True
    kernel_backend: str = "b200"
    kernel_mode: str = "fast"
    decay_init_bias: float = 3.0
    rope_base: float = 10000.0
    global_rel_pos_dim: int = 64
    annealing_enabled: bool = True
    T_start: float = 10.0
    T_end: float = 0.1
    annealing_steps: int = 1000
    annealing_schedule: str = "cosine"
    quantum_tunneling_enabled: bool = False
    tunneling_strength: float = 0.1
    num_tunnel_paths: int = 4
    energy_landscape: str = "entropy"
    tunneling_schedule: str = "adaptive"

    def to_dict(self) -> Dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, config_dict: Dict) -> "TESMConfig":
        return cls(**{k: v for k, v in config_dict.items() if k in cls.__dataclass_fields__})


@dataclass
class TESMCausalLMOutput:
    loss: Optional[torch.Tensor] = None
    logits: Optional[torch.Tensor] = None
    hidden_states: Optional[torch.Tensor] = None
    entanglement_maps: Optional[List[torch.Tensor]] = None
    entanglement_stats: Optional[Dict[str, float]] = None


class FeedForward(nn.Module):
    """SwiGLU-style FFN of ternary BitLinears (mixer_seq_simple.py:25-67)."""

    def __init__(self, config: TESMConfig, device=None, dtype=None):
        super().__init__()
        fk = {"device": device, "dtype": dtype}
        bl = dict(bias=False, bit_eps=config.bit_eps, bit_threshold=config.bit_threshold,
                  kernel_backend=config.kernel_backend, kernel_mode=config.kernel_mode, **fk)
        self.gate_proj = BitLinear(config.d_model, config.d_intermediate, **bl)
        self.up_proj = BitLinear(config.d_model, config.d_intermediate, **bl)
        self.down_proj = BitLinear(config.d_intermediate, config.d_model, **bl)
        self.dropout = nn.Dropout(config.dropout)

    def forward(self, x):
        return layers.ffn_forward(self, x)


class MixerModel(nn.Module):
    """Embedding + TESM blocks + final norm (mixer_seq_simple.py:70-242)."""

    def __init__(self, config: TESMConfig, device=None, dtype=None):
        super().__init__()
        fk = {"device": device, "dtype": dtype}
        self.config = config
        self.gradient_checkpointing = config.gradient_checkpointing
        self.residual_in_fp32 = config.residual_in_fp32
        self.embedding = nn.Embedding(config.vocab_size, config.d_model, **fk)
        self.position_embedding = nn.Embedding(config.max_seq_len, config.d_model, **fk)
        norm_cls = partial(RMSNorm if config.rms_norm else nn.LayerNorm, eps=config.norm_epsilon)
        if config.use_mimo:
            def mixer_cls(layer_idx):
                return lambda dim: TESMMIMO_Optimized(
                    d_model=dim, n_heads=config.n_heads, d_state=config.d_state, expand=config.expand,
                    ent_rank=config.ent_rank, entanglement_window=config.entanglement_window,
                    entanglement_threshold=config.entanglement_threshold,
                    entanglement_scale=config.entanglement_scale, max_seq_len=config.max_seq_len,
                    dropout=config.dropout, bit_eps=config.bit_eps, bit_threshold=config.bit_threshold,
                    kernel_backend=config.kernel_backend, annealing_enabled=config.annealing_enabled,
                    T_start=config.T_start, T_end=config.T_end, annealing_steps=config.annealing_steps,
                    annealing_schedule=config.annealing_schedule, **fk)
        else:
            def mixer_cls(layer_idx):
                return lambda dim: TESM_SISO(
                    d_model=dim, d_state=config.d_state, expand=config.expand, ent_rank=config.ent_rank,
                    entanglement_scale=config.entanglement_scale,
                    entanglement_threshold=config.entanglement_threshold,
                    entanglement_window=config.entanglement_window,
                    entanglement_block_size=config.entanglement_block_size,
                    entanglement_init=config.entanglement_init, layer_idx=layer_idx,
                    max_seq_len=config.max_seq_len, dropout=config.dropout, bit_eps=config.bit_eps,
                    bit_threshold=config.bit_threshold, kernel_backend=config.kernel_backend,
                    kernel_mode=config.kernel_mode, use_triton_kernels=config.use_triton_kernels,
                    state_scan_chunk_size=config.state_scan_chunk_size, decay_init_bias=config.decay_init_bias,
                    rope_base=getattr(config, "rope_base", 10000.0), annealing_enabled=config.annealing_enabled,
                    T_start=config.T_start, T_end=config.T_end, annealing_steps=config.annealing_steps,
                    annealing_schedule=config.annealing_schedule,
                    quantum_tunneling_enabled=config.quantum_tunneling_enabled,
                    tunneling_strength=config.tunneling_strength, num_tunnel_paths=config.num_tunnel_paths,
                    energy_landscape=config.energy_landscape, tunneling_schedule=config.tunneling_schedule, **fk)
        mlp_cls = lambda dim: FeedForward(config, device=device, dtype=dtype)  # noqa: E731
        self.layers = nn.ModuleList([
            Block(config.d_model, mixer_cls(i), mlp_cls, norm_cls=norm_cls, residual_in_fp32=config.residual_in_fp32)
            for i in range(config.n_layer)])
        for i, layer in enumerate(self.layers):
            layer.layer_idx = i
        self.norm_f = (RMSNorm if config.rms_norm else nn.LayerNorm)(config.d_model, eps=config.norm_epsilon)
        self.apply(partial(_init_weights, n_layer=config.n_layer, initializer_range=config.initializer_range,
                           rescale_prenorm_residual=config.rescale_prenorm_residual, n_residuals_per_layer=1))

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kwargs):
        return {i: layer.allocate_inference_cache(batch_size, max_seqlen, dtype=dtype, **kwargs)
                for i, layer in enumerate(self.layers)}

    def forward(self, input_ids, inference_params=None, prev_states=None, **mixer_kwargs):
        return layers.mixer_model_forward(self, input_ids, inference_params, prev_states, **mixer_kwargs)


class TESMLMHeadModel(nn.Module):
    """Causal LM head over the mixer (mixer_seq_simple.py:245-345)."""

    def __init__(self, config: Optional[TESMConfig] = None, device=None, dtype=None):
        super().__init__()
        self.tesm_config = config or TESMConfig()
        config = self.tesm_config
        self.backbone = MixerModel(config, device=device, dtype=dtype)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False, device=device, dtype=dtype)
        if config.tie_embeddings:
            self.lm_head.weight = self.backbone.embedding.weight
        self.vocab_suppression = getattr(config, "vocab_suppression", False)
        self.suppression_bias = getattr(config, "suppression_bias", -10.0)
        self.semantic_activation = getattr(config, "semantic_activation", False)
        self.semantic_activation_strength = getattr(config, "semantic_activation_strength", 0.5)
        self.semantic_activation_threshold = getattr(config, "semantic_activation_threshold", 0.3)
        self.cooccurrence_topk = getattr(config, "cooccurrence_topk", 100)
        if self.semantic_activation:
            self.register_buffer("related_token_ids", torch.zeros(config.vocab_size, self.cooccurrence_topk,
                                                                  dtype=torch.long))
            self.register_buffer("related_token_strengths", torch.zeros(config.vocab_size, self.cooccurrence_topk,
                                                                        dtype=torch.float32))
            self.register_buffer("token_freq", torch.zeros(config.vocab_size, dtype=torch.float32))
            self.cooccurrence_built = False

    def get_input_embeddings(self):
        return self.backbone.embedding

    def set_input_embeddings(self, value):
        self.backbone.embedding = value
        if self.tesm_config.tie_embeddings:
            self.lm_head.weight = value.weight

    def forward(self, input_ids, labels=None, inference_params=None, prev_states=None, logits_to_keep: int = 0,
                sparse_logits: bool = False, **kwargs):
        for k in ["attention_mask", "past_key_values", "use_cache"]:
            kwargs.pop(k, None)
        return layers.lm_forward(self, input_ids, labels, inference_params, prev_states, logits_to_keep, **kwargs)

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens: int = 64, temperature: float = 1.0, top_k: int = 0,
                 use_cache: bool = True, sparse_inference: bool = False, dynamic_activation: bool = True,
                 use_graph=None):
        """Token generation with the recurrent-state cache (mixer_seq_simple.py:617-703); the
        incremental steps replay a captured CUDA graph.  ``sparse_inference`` /
        ``dynamic_activation`` only act with vocabulary suppression, which is outside the b200
        path (this model raises for it), so they are accepted and have no effect."""
        return layers.generate(self, input_ids, max_new_tokens, temperature, top_k, use_cache, use_graph)


def _init_weights(module, n_layer, initializer_range=0.02, rescale_prenorm_residual=True, n_residuals_per_layer=1):
    """Seeded init of mixer_seq_simple.py:790-803.

    The reference's residual rescale compares non-recursive parameter names
    ("weight") with "out_proj.weight"/"down_proj.weight" and so never fires; this
    mirror keeps that behaviour so seeded weights match.
    """
    if isinstance(module, nn.Linear):
        if module.bias is not None:
            nn.init.zeros_(module.bias)
        nn.init.normal_(module.weight, std=initializer_range)
    elif isinstance(module, BitLinear):
        nn.init.normal_(module.weight, std=initializer_range)
    elif isinstance(module, nn.Embedding):
        nn.init.normal_(module.weight, std=initializer_range)
    if rescale_prenorm_residual:
        for name, param in module.named_parameters(recurse=False):
            if name in ["out_proj.weight", "down_proj.weight"]:
                with torch.no_grad():
                    param /= (n_residuals_per_layer * n_layer) ** 0.5
