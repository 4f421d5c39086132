"""The reference's causal LM around the kernels: the caller of the hot path at model scale.

Mirrors src/prime_moment_attention/model.py (PrimeConfig :20-44, RMSNorm :47-56, PrimeMLP :59-68,
PrimeBlock :71-117, PrimeForCausalLM :120-244) with the same parameter names and shapes, so a
state_dict of the reference model loads unchanged; every attention layer is this package's
PrimeMomentAttention (prologue and core on the CUDA kernels).  Inference only.

Beyond the reference's forward / generate, two serving paths:
  * forward(..., last_logits_only=True) computes the LM head for the last position only (what
    generate needs; the reference computes [B, L, vocab] logits);
  * DecodeGraph: one greedy decode step of the whole model captured in a CUDA graph, the
    per-layer states updated in place by pma_decode_step (no Python or allocation per step).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .attention import PrimeMomentAttention, _prologue
from .selective import PrimeSelectiveMomentAttention


@dataclass
class PrimeConfig:
    """Same fields and defaults as the reference PrimeConfig (model.py:20-44)."""
    vocab_size: int = 32000
    hidden_size: int = 512
    num_layers: int = 6
    num_heads: int = 8
    head_dim: int = 64
    num_kv_heads: Optional[int] = None
    intermediate_size: Optional[int] = None
    decay: float = 0.9995
    use_qk_norm: bool = True
    rms_norm_eps: float = 1e-6
    eps: float = 1.0
    tie_word_embeddings: bool = True
    initializer_range: float = 0.02
    use_selective: bool = False
    min_tau: float = 2.0
    max_tau: float = 2000.0

    def __post_init__(self):
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads
        if self.intermediate_size is None:
            self.intermediate_size = int(2 * (4 * self.hidden_size) / 3)


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight (model.py:47-56), as torch's fused rms_norm."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


class PrimeMLP(nn.Module):
    """SwiGLU feed-forward (model.py:59-68); silu(gate) * up as one kernel (pma_swiglu)."""

    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(ops.swiglu(self.gate_proj(x), self.up_proj(x)))


class PrimeBlock(nn.Module):
    """Pre-norm block (model.py:71-117)."""

    def __init__(self, config: PrimeConfig):
        super().__init__()
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        if config.use_selective:
            self.self_attn = PrimeSelectiveMomentAttention(
                hidden_size=config.hidden_size, num_heads=config.num_heads, head_dim=config.head_dim,
                num_kv_heads=config.num_kv_heads, decay=config.decay, use_qk_norm=config.use_qk_norm,
                eps=config.eps, min_tau=config.min_tau, max_tau=config.max_tau)
        else:
            self.self_attn = PrimeMomentAttention(hidden_size=config.hidden_size, num_heads=config.num_heads,
                                                  head_dim=config.head_dim, num_kv_heads=config.num_kv_heads,
                                                  decay=config.decay, use_qk_norm=config.use_qk_norm,
                                                  eps=config.eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.mlp = PrimeMLP(config.hidden_size, config.intermediate_size)

    def forward(self, hidden_states, state=None, return_state=False):
        residual = hidden_states
        hidden_states, next_state = self.self_attn(self.input_layernorm(hidden_states), state=state,
                                                   return_state=return_state)
        hidden_states = residual + hidden_states
        hidden_states = hidden_states + self.mlp(self.post_attention_layernorm(hidden_states))
        return hidden_states, next_state


class PrimeForCausalLM(nn.Module):
    """Decoder-only LM (model.py:120-244); attention on the CUDA kernels."""

    def __init__(self, config: PrimeConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([PrimeBlock(config) for _ in range(config.num_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.embed_tokens.weight
        self.apply(self._init_weights)
        scale = config.initializer_range / math.sqrt(2 * config.num_layers)
        with torch.no_grad():
            for layer in self.layers:
                layer.self_attn.o_proj.weight.normal_(mean=0.0, std=scale)
                layer.mlp.down_proj.weight.normal_(mean=0.0, std=scale)
                if hasattr(layer.self_attn, "init_selective_weights"):
                    layer.self_attn.init_selective_weights()

    def _init_weights(self, module: nn.Module):
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=self.config.initializer_range)
            if getattr(module, "bias", None) is not None:
                nn.init.zeros_(module.bias)

    def get_input_embeddings(self) -> nn.Embedding:
        return self.embed_tokens

    def forward(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None,
                states: Optional[List[Tuple[torch.Tensor, ...]]] = None, return_states: bool = False,
                last_logits_only: bool = False) -> Dict[str, Any]:
        hidden_states = self.embed_tokens(input_ids)
        next_states = [] if return_states else None
        for i, layer in enumerate(self.layers):
            hidden_states, next_s = layer(hidden_states, state=states[i] if states is not None else None,
                                          return_state=return_states)
            if return_states:
                next_states.append(next_s)
        if last_logits_only:
            hidden_states = hidden_states[:, -1:]
        logits = self.lm_head(self.norm(hidden_states))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[..., :-1, :].float().reshape(-1, self.config.vocab_size),
                                   labels[..., 1:].reshape(-1), ignore_index=-100)
        return {"loss": loss, "logits": logits, "states": next_states}

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 50, temperature: float = 1.0,
                 top_k: int = 50, eos_token_id: Optional[int] = None) -> torch.Tensor:
        """Same sampling rule as model.py:203-242 (greedy when temperature == 0)."""
        self.eval()
        out = self.forward(input_ids, return_states=True, last_logits_only=True)
        states, logits = out["states"], out["logits"][:, -1, :]
        generated = input_ids
        for _ in range(max_new_tokens):
            logits = torch.nan_to_num(logits, nan=0.0, posinf=50.0, neginf=-50.0)
            if temperature > 0.0:
                lg = logits / max(temperature, 1e-4)
                if top_k > 0:
                    v, _ = torch.topk(lg, min(top_k, lg.size(-1)))
                    lg[lg < v[:, [-1]]] = -float("Inf")
                probs = torch.nan_to_num(F.softmax(lg, dim=-1), nan=1.0 / self.config.vocab_size)
                nxt = torch.multinomial(probs, num_samples=1)
            else:
                nxt = torch.argmax(logits, dim=-1, keepdim=True)
            generated = torch.cat([generated, nxt], dim=-1)
            if eos_token_id is not None and (nxt == eos_token_id).all():
                break
            out = self.forward(nxt, states=states, return_states=True)
            states, logits = out["states"], out["logits"][:, -1, :]
        return generated


class DecodeGraph:
    """One greedy decode step of `model` for a fixed batch, captured in a CUDA graph.

    The per-layer states are owned here (copied from `states` once) and updated in place by
    pma_decode_step_ex (pma_selective_decode_step for selective layers, whose per-token decay is
    computed inside the graph); `step()` replays the graph: token ids in `self.tokens` [B, 1] ->
    next greedy ids in `self.tokens` and the step's logits in `self.logits` [B, vocab].
    Mirrors the decode loop of generate (model.py:227-240) with temperature 0."""

    def __init__(self, model: PrimeForCausalLM, states: List[Tuple[torch.Tensor, ...]], tokens: torch.Tensor,
                 warmup: int = 2):
        self.model = model
        dev = tokens.device
        self.states = [tuple(t.detach().to(torch.float32).contiguous().clone() for t in st) for st in states]
        # one GEMM for q, k, v and one for gate, up per layer (concatenated copies of the weights,
        # taken now: the graph serves the weights as they are at construction)
        self.w_qkv, self.w_gu = [], []
        for layer in model.layers:
            a, mlp = layer.self_attn, layer.mlp
            self.w_qkv.append(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight]).detach().contiguous())
            self.w_gu.append(torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]).detach().contiguous())
        self.tokens = tokens.detach().reshape(-1, 1).clone()
        self.logits = None
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):  # settles allocator pools and per-module caches before capture
                self._body(write=False)
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body(write=True)

    def _body(self, write: bool):
        m = self.model
        h = m.embed_tokens(self.tokens)  # [B, 1, hidden]
        h = h[:, 0]  # [B, hidden]
        for layer, st, w_qkv, w_gu in zip(m.layers, self.states, self.w_qkv, self.w_gu):
            attn = layer.self_attn
            x = layer.input_layernorm(h)
            B = x.shape[0]
            H, D, Hk = attn.num_heads, attn.head_dim, attn.num_kv_heads
            qkv = torch.mm(x, w_qkv.t())  # [B, (H + 2 Hk) D]; q, k, v are strided views of it
            q = qkv[:, :H * D].view(B, H, D)
            k = qkv[:, H * D:(H + Hk) * D].view(B, Hk, D)
            v = qkv[:, (H + Hk) * D:].view(B, Hk, D)
            pro = _prologue(attn)
            if pro is None:
                raise NotImplementedError("DecodeGraph needs QK-norms the kernels fold (nn.LayerNorm over head_dim)")
            st_step = st if write else tuple(t.clone() for t in st)
            if isinstance(attn, PrimeSelectiveMomentAttention):
                # this token's decay exp(-Delta / tau_h), Delta = clamp(softplus(delta_proj(x)), 1e-4, 50),
                # and k scaled by beta_h, as in the step branch (selective.py:367-396)
                delta = F.softplus(attn.delta_proj(x)).clamp(min=1e-4, max=50.0)  # [B, H]
                log_decay = -delta.float() / attn.get_tau(x.device).view(1, H)
                y, _ = ops.selective_decode_step(q, k, v, log_decay, attn.get_beta(x.device).float(), st_step,
                                                 eps=attn.eps, inplace=True, prologue=pro)
            else:
                decay = getattr(attn, "decay_per_head", None)
                decay = attn.decay if decay is None else decay
                y, _ = ops.decode_step(q, k, v, decay, st_step, eps=attn.eps, inplace=True, prologue=pro)
            h = torch.addmm(h, y.reshape(B, H * D).to(h.dtype), attn.o_proj.weight.t())  # residual + o_proj
            gu = torch.mm(layer.post_attention_layernorm(h), w_gu.t())
            inter = gu.shape[1] // 2
            h = torch.addmm(h, ops.swiglu(gu[:, :inter], gu[:, inter:]), layer.mlp.down_proj.weight.t())
        logits = m.lm_head(m.norm(h))
        nxt = torch.argmax(logits, dim=-1, keepdim=True)
        if write:
            self.logits = logits
            self.tokens.copy_(nxt)

    def step(self) -> torch.Tensor:
        self.graph.replay()
        return self.tokens
