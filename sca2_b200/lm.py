"""Language model on the layer protocol (the role of lapa/model.py:24-109), a training step,
and decoding with the whole stack's single-token step captured in one CUDA graph.

    LM(layer_factory, n_layers, vocab, d, tie_embeddings=False)
        forward(tokens) -> logits; prefill(tokens, state) -> (logits, state);
        step(token, state) -> (logits, state); generate(prompt, n, ...) -> ids
    LaplaceLM(vocab, d, n_layers, **LaplaceConfig fields)   lapa/model.py LaplaceLM
    GatedLM(vocab, cfg: LayerCfg, n_layers)                 GatedLayer stack (multi-head SCA2)
    GraphDecoder(lm, B)                                     CUDA-graph decode (sca2/decode.py:55-108)
    zipf_tokens(n, vocab, s, seed), train_step(...)

Parameter names follow the reference (embed, layers.i, norm, head), so a reference LM's
state_dict loads with strict=True.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .heads import LaplaceConfig
from .layers import GatedLayer, LaplaceAttention, LayerCfg, LayerNorm


class LM(nn.Module):
    """Token embedding -> a stack of protocol layers -> final LayerNorm -> vocabulary projection.

    Any layer with the prefill / step / init_state protocol stacks here (layer_factory(i)
    builds layer i).  Parameter names (embed, layers.<i>, norm, head) and the optional tying
    of the head to the embedding are those of lapa/model.py, so a reference LM's state_dict
    loads with strict=True; the decode state is the list of the layers' states."""

    def __init__(self, layer_factory: Callable[[int], nn.Module], n_layers: int, vocab: int, d: int,
                 tie_embeddings: bool = False):
        super().__init__()
        self.d, self.vocab = d, vocab
        self.embed = nn.Embedding(vocab, d)
        self.layers = nn.ModuleList(layer_factory(i) for i in range(n_layers))
        self.norm = LayerNorm(d)
        self.head = nn.Linear(d, vocab, bias=False)
        if tie_embeddings:
            self.head.weight = self.embed.weight

    def init_state(self, B: int, device) -> List[Dict]:
        return [layer.init_state(B, device) for layer in self.layers]

    def _through(self, x: torch.Tensor, state: List[Dict], method: str):
        """Run x through every layer's `method` ("prefill" or "step"); the layers' new states."""
        new = []
        for layer, st in zip(self.layers, state):
            x, st = getattr(layer, method)(x, st)
            new.append(st)
        return self.head(self.norm(x)), new

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.prefill(tokens)[0]

    def prefill(self, tokens: torch.Tensor, state: Optional[List[Dict]] = None):
        """tokens (B,T) -> logits (B,T,vocab) and the state after the last token."""
        state = state if state is not None else self.init_state(tokens.size(0), tokens.device)
        return self._through(self.embed(tokens), state, "prefill")

    def step(self, token: torch.Tensor, state: List[Dict]):
        """token (B,) -> logits (B,vocab) and the advanced state."""
        return self._through(self.embed(token), state, "step")

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, n: int, temperature: float = 1.0, top_k: int = 0,
                 greedy: bool = False) -> torch.Tensor:
        """Prefill the prompt ((B,T) or (T,) ids), then n decode steps; returns the prompt with
        the n new ids appended, in the prompt's layout (the contract of lapa/model.py:68-95)."""
        ids = prompt if prompt.dim() == 2 else prompt.unsqueeze(0)
        logits, state = self.prefill(ids)
        last, picked = logits[:, -1], []
        for _ in range(n):
            tok = next_token(last, temperature, top_k, greedy)
            picked.append(tok)
            last, state = self.step(tok, state)
        out = torch.cat([ids, torch.stack(picked, 1)], 1) if picked else ids
        return out if prompt.dim() == 2 else out[0]

    def layer_params(self) -> int:
        return sum(p.numel() for p in self.layers.parameters())

    def state_floats(self) -> Optional[int]:
        """Decode-state floats per sequence over all layers, or None when a layer does not
        report a fixed size."""
        sizes = [getattr(layer, "state_floats", lambda: None)() for layer in self.layers]
        return None if any(v is None for v in sizes) else sum(sizes)


def next_token(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0, greedy: bool = False) -> torch.Tensor:
    """(B, vocab) logits -> (B,) ids: the arg-max when greedy (or temperature <= 0), else a draw
    from softmax(logits / temperature), restricted to the top_k most likely ids when top_k > 0."""
    if greedy or temperature <= 0:
        return logits.argmax(-1)
    probs = torch.softmax(logits.float() / temperature, -1)
    if not top_k or top_k >= probs.size(-1):
        return torch.multinomial(probs, 1).squeeze(-1)
    top_p, top_i = probs.topk(top_k, -1)
    return top_i.gather(-1, torch.multinomial(top_p, 1)).squeeze(-1)


class LaplaceLM(LM):
    """lapa/model.py LaplaceLM: LaplaceAttention layers with LaplaceConfig(d=d, **cfg)."""

    def __init__(self, vocab: int, d: int = 128, n_layers: int = 4, tie_embeddings: bool = False, **cfg):
        c = LaplaceConfig(d=d, **cfg)
        super().__init__(lambda i: LaplaceAttention(c), n_layers, vocab, d, tie_embeddings)


class GatedLM(LM):
    """A stack of GatedLayer (multi-head gated SCA2 layers, sca2/arch_gatedc.py:199-256)."""

    def __init__(self, vocab: int, cfg: LayerCfg, n_layers: int = 12, tie_embeddings: bool = False):
        super().__init__(lambda i: GatedLayer(cfg), n_layers, vocab, cfg.d, tie_embeddings)


def init_weights(model: nn.Module, std: float = 0.02):
    """Random init with N(0, std^2) for every Linear / Embedding weight (biases zero), the
    LM benchmark's initialisation; head parameters that are not matrices keep their init."""
    for m in model.modules():
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, 0.0, std)
            if getattr(m, "bias", None) is not None:
                nn.init.zeros_(m.bias)


# ------------------------------------------------------------------------------------------
#  CUDA-graph decode
# ------------------------------------------------------------------------------------------
def _tree_copy_(dst, src):
    if isinstance(dst, dict):
        for k in dst:
            _tree_copy_(dst[k], src[k])
    elif isinstance(dst, (list, tuple)):
        for a, b in zip(dst, src):
            _tree_copy_(a, b)
    elif torch.is_tensor(dst):
        dst.copy_(src)


def _tree_clone(x):
    if isinstance(x, dict):
        return {k: _tree_clone(v) for k, v in x.items()}
    if isinstance(x, list):
        return [_tree_clone(v) for v in x]
    if isinstance(x, tuple):
        return tuple(_tree_clone(v) for v in x)
    return x.clone() if torch.is_tensor(x) else x


class GraphDecoder:
    """One decode step of the whole stack (embedding, every layer's step, norm, head, greedy
    pick) captured once in a CUDA graph over static token / state buffers, then replayed per
    token (the role of sca2/decode.py:55-108).  The states are copied into the static buffers
    inside the graph, so a replay advances every layer's state in place."""

    def __init__(self, lm: LM, state: List[Dict], warmup: int = 2):
        self.lm = lm
        B = _batch_of(state)
        dev = next(lm.parameters()).device
        self.tok = torch.zeros(B, dtype=torch.long, device=dev)
        self.state = _tree_clone(state)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):   # warm-up on a copy: the real state must not advance
                tmp = _tree_clone(self.state)
                lm.step(self.tok, tmp)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            logits, new = lm.step(self.tok, self.state)
            self.next_tok = logits.argmax(-1)
            self.logits = logits
            _tree_copy_(self.state, new)

    def step(self, tok: torch.Tensor) -> torch.Tensor:
        self.tok.copy_(tok)
        self.graph.replay()
        return self.next_tok

    @torch.no_grad()
    def generate(self, first: torch.Tensor, n: int) -> torch.Tensor:
        """Greedy: n tokens after `first` (B,), each from one graph replay."""
        out, tok = [], first
        for _ in range(n):
            tok = self.step(tok).clone()
            out.append(tok)
        return torch.stack(out, 1)


def _batch_of(state):
    for s in state:
        for v in _leaves(s):
            if torch.is_tensor(v) and v.dim() >= 1:
                return v.size(0)
    raise ValueError("no batched tensor in the state")


def _leaves(x):
    if isinstance(x, dict):
        for v in x.values():
            yield from _leaves(v)
    elif isinstance(x, (list, tuple)):
        for v in x:
            yield from _leaves(v)
    else:
        yield x


# ------------------------------------------------------------------------------------------
#  training
# ------------------------------------------------------------------------------------------
def zipf_tokens(n_seq: int, T: int, vocab: int, s: float = 1.1, seed: int = 0, device="cpu") -> torch.Tensor:
    """(n_seq, T) token ids: ranks drawn Zipf(s) over [1, vocab], mapped to ids by a seeded
    permutation (the LM benchmark's synthetic corpus)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    p = torch.arange(1, vocab + 1, dtype=torch.float64) ** (-s)
    ranks = torch.multinomial((p / p.sum()).float(), n_seq * T, replacement=True, generator=g)
    perm = torch.randperm(vocab, generator=g)
    return perm[ranks].view(n_seq, T).to(device)


def lm_loss(model: nn.Module, tokens: torch.Tensor) -> torch.Tensor:
    """Next-token cross entropy over tokens (B, T+1)."""
    logits = model(tokens[:, :-1])
    return F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), tokens[:, 1:].reshape(-1))


def train_step(model: nn.Module, opt: torch.optim.Optimizer, tokens: torch.Tensor,
               dtype: Optional[torch.dtype] = torch.bfloat16) -> torch.Tensor:
    """One optimizer step (bf16 autocast by default); returns the loss (device scalar)."""
    with torch.autocast("cuda", dtype=dtype, enabled=dtype is not None):
        loss = lm_loss(model, tokens)
    loss.backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return loss.detach()
