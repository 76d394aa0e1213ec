"""Qwen3 decoding over the tree-shared KV pool (reference ``src/tree_attention/qwen.py:9-124``).

``SharedKVDecoder(model, sequences, max_new_tokens=32, method="cube",
cost_model=None)`` keeps ONE physical copy of every shared prefix per layer and
runs each decode step's attention through ``attention_matrix`` (looked up as a
module global at call time, so a caller may substitute it, as the reference's
model checks do).  ``CachedPrefixDecoder`` schedules the prompt once and only
rewrites the lengths of the private decode tails each step
(``CachedDecodePlan``).  Both expose the reference's attributes: ``logits``,
``tree``, ``sequences``, ``used``, ``capacity``, ``prefix_size``,
``max_new_tokens``, ``generated`` and, for the cached decoder, ``cached_plan``.

Differences from the reference, on purpose:

* pools are ``[HK, capacity, D]`` for K and V alike (the kernels' token-major
  layout; the reference keeps K as ``[HK, D, capacity]``);
* ``prefill="shared"`` (default) computes every tree node's K/V once, feeding
  the node's tokens with its ancestors' K/V as the attention cache, instead of
  one full forward per request (``prefill="per_request"`` is the reference's
  procedure, ``qwen.py:34-51``); logits of a request are those at the last
  token of its terminal node;
* ``shard=(rank, world, group)`` splits the KV heads over GPUs (each rank owns
  ``HK / world`` KV heads and their query heads, the matching slices of the
  q/k/v projections and its slice of every pool) and all-gathers the attention
  outputs (NCCL ``all_gather_into_tensor``) before ``o_proj``; the plan is the
  same on every rank.
"""
from __future__ import annotations

from types import MethodType

import torch

from .kernels import CachedDecodePlan, append_kv, attention_matrix, prepare
from .schedule import CostModel, schedule
from .tree import KVTree

try:
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb
except ImportError:                                   # transformers without Qwen3
    apply_rotary_pos_emb = None


def _rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def _rope(q, k, cos, sin):
    if apply_rotary_pos_emb is not None:
        return apply_rotary_pos_emb(q, k, cos, sin)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


class SharedKVDecoder:
    """Qwen3 decode with one physical shared-prefix KV pool per layer (reference qwen.py:9-103)."""

    def __init__(self, model, sequences, max_new_tokens=32, method="cube", cost_model=None, prefill="shared",
                 shard=None):
        if prefill not in ("shared", "per_request"):
            raise ValueError(f"unknown prefill {prefill!r}")
        self.model = model
        self.sequences = [list(s) for s in sequences]
        if not self.sequences or any(not s for s in self.sequences):
            raise ValueError("every sequence needs at least one token")
        self.tree = KVTree.from_sequences(self.sequences)
        self.method = method
        self.cost_model = cost_model or CostModel()
        self.device = next(model.parameters()).device
        config = model.config
        self.hq, self.hk = config.num_attention_heads, config.num_key_value_heads
        self.dim = getattr(config, "head_dim", None) or config.hidden_size // self.hq
        self.rank, self.world, self.group = shard if shard is not None else (0, 1, None)
        if self.hk % self.world:
            raise ValueError(f"{self.hk} KV heads do not split over {self.world} GPUs")
        self.local_hk = self.hk // self.world
        self.local_hq = self.hq // self.world
        self.original = [layer.self_attn.forward for layer in model.model.layers]
        self.max_new_tokens = max_new_tokens
        self.capacity = self.tree.storage_tokens + len(self.sequences) * max_new_tokens
        self.used = self.tree.storage_tokens
        self.prefix_size = self.used
        self.generated = 0
        self.pools = [(torch.empty((self.local_hk, self.capacity, self.dim), device=self.device, dtype=model.dtype),
                       torch.empty((self.local_hk, self.capacity, self.dim), device=self.device, dtype=model.dtype))
                      for _ in model.model.layers]
        self.leaves = [next(i for i, n in enumerate(self.tree.nodes) if r in n.terminal)
                       for r in range(len(self.sequences))]
        self._slices = self._projection_slices()
        if prefill == "shared":
            self._prefill_shared()
        else:
            self._prefill_per_request()

    # -- head sharding ----------------------------------------------------------
    def _projection_slices(self):
        """Row slices of q/k/v projection weights owned by this rank (None: all)."""
        if self.world == 1:
            return None
        q0 = self.rank * self.local_hq * self.dim
        k0 = self.rank * self.local_hk * self.dim
        return (slice(q0, q0 + self.local_hq * self.dim), slice(k0, k0 + self.local_hk * self.dim))

    # -- prefill ----------------------------------------------------------------
    @torch.inference_mode()
    def _prefill_per_request(self):
        """One full forward per request; copy positions not written yet (reference qwen.py:34-51)."""
        assigned, logits = set(), []
        for request, seq in enumerate(self.sequences):
            output = self.model(torch.tensor([seq], device=self.device), use_cache=True)
            logits.append(output.logits[0, -1].clone())
            path = self.tree.paths[request]
            fresh = [i for i, position in enumerate(path) if position not in assigned]
            if fresh:
                source = torch.tensor(fresh, device=self.device)
                target = torch.tensor([path[i] for i in fresh], device=self.device)
                for layer, (kp, vp) in zip(self._cache_layers(output.past_key_values), self.pools):
                    keys, values = layer
                    kp.index_copy_(1, target, self._local_kv(keys[0]).index_select(1, source))
                    vp.index_copy_(1, target, self._local_kv(values[0]).index_select(1, source))
            assigned.update(path)
        self.logits = torch.stack(logits)

    @torch.inference_mode()
    def _prefill_shared(self):
        """Every tree node once, its ancestors' K/V as the cache (shared-prefix prefill)."""
        from transformers import DynamicCache
        nodes = self.tree.nodes
        node_logits = {}
        # full KV of every node, all heads, kept until its subtree is done (depth-first order)
        full_kv = {}
        children_left = {i: len(n.children) for i, n in enumerate(nodes)}
        order = [i for i in range(len(nodes))]           # nodes are created parent before child
        for i in order:
            node = nodes[i]
            if not node.tokens:                           # the empty root
                continue
            chain = []
            a = node.parent
            while a is not None and a >= 0:
                chain.append(a)
                a = nodes[a].parent
            chain.reverse()
            chain = [a for a in chain if nodes[a].tokens]
            offset = sum(len(nodes[a].tokens) for a in chain)
            tokens = torch.tensor([self.tree.token_ids[p] for p in node.tokens], device=self.device)[None]
            cache = None
            if chain:
                cache = DynamicCache()
                for layer_idx in range(len(self.pools)):
                    keys = torch.cat([full_kv[a][layer_idx][0] for a in chain], dim=2)
                    values = torch.cat([full_kv[a][layer_idx][1] for a in chain], dim=2)
                    cache.update(keys, values, layer_idx)
            positions = torch.arange(offset, offset + tokens.shape[1], device=self.device)[None]
            output = self.model(tokens, past_key_values=cache, position_ids=positions, use_cache=True)
            layers = list(self._cache_layers(output.past_key_values))
            fresh = [(keys[:, :, offset:], values[:, :, offset:]) for keys, values in layers]
            full_kv[i] = fresh
            target = torch.tensor(node.tokens, device=self.device)
            for (keys, values), (kp, vp) in zip(fresh, self.pools):
                kp.index_copy_(1, target, self._local_kv(keys[0]))
                vp.index_copy_(1, target, self._local_kv(values[0]))
            node_logits[i] = output.logits[0, -1].clone()
            # release K/V of finished subtrees
            a = node.parent
            if not node.children:
                full_kv.pop(i, None)
                while a is not None and a >= 0:
                    children_left[a] -= 1
                    if children_left[a]:
                        break
                    full_kv.pop(a, None)
                    a = nodes[a].parent
        self.logits = torch.stack([node_logits[leaf] for leaf in self.leaves])

    def _cache_layers(self, cache):
        """(keys, values) per layer of a transformers cache, [1, HK, T, D] each."""
        if hasattr(cache, "layers"):
            return [(layer.keys, layer.values) for layer in cache.layers]
        return [(cache.key_cache[i], cache.value_cache[i]) for i in range(len(cache.key_cache))]

    def _local_kv(self, states):
        """[HK, T, D] -> this rank's KV heads."""
        if self.world == 1:
            return states
        return states[self.rank * self.local_hk:(self.rank + 1) * self.local_hk]

    # -- decode -----------------------------------------------------------------
    def _next_positions(self, count):
        positions = [self.prefix_size + r * self.max_new_tokens + self.generated for r in range(count)]
        self.generated += 1
        return positions

    def _prepare_plan(self):
        plan = schedule(self.tree, self.hq, self.hk, self.dim, self.method, self.cost_model)
        q = torch.empty((len(self.sequences), self.local_hq, self.dim), device=self.device, dtype=self.model.dtype)
        return prepare(plan, q, self.local_hk)

    def _append(self, token_ids):
        if self.used + len(token_ids) > self.capacity:
            raise ValueError("Decode exceeds allocated max_new_tokens")
        positions = self._next_positions(len(token_ids))
        for sequence, token in zip(self.sequences, token_ids):
            sequence.append(token)
        self.tree.extend_leaves(self.leaves, positions)
        self.used += len(token_ids)
        return positions

    def _attention_forward(self, prepared, targets, nreq, tails=None):
        """The decode-step attention of every layer: q/k/v projections (this rank's heads), q/k RMSNorm,
        RoPE, append of the new K/V at ``targets`` (a device tensor of pool positions) by one fused launch,
        tree attention through ``attention_matrix`` and, when sharded, an all-gather of the heads before
        ``o_proj``.  ``tails = (cached_plan, count, offset)`` lets the first layer's append also set the
        plan's tail lengths to ``count + offset`` on the device."""
        pools, slices, decoder = self.pools, self._slices, self

        def forward(module, hidden_states, position_embeddings, attention_mask=None, **kwargs):
            shape = (*hidden_states.shape[:-1], -1, module.head_dim)
            if slices is None:
                q = module.q_proj(hidden_states)
                k = module.k_proj(hidden_states)
                v = module.v_proj(hidden_states)
            else:
                qs, ks = slices
                q = torch.nn.functional.linear(hidden_states, module.q_proj.weight[qs],
                                               None if module.q_proj.bias is None else module.q_proj.bias[qs])
                k = torch.nn.functional.linear(hidden_states, module.k_proj.weight[ks],
                                               None if module.k_proj.bias is None else module.k_proj.bias[ks])
                v = torch.nn.functional.linear(hidden_states, module.v_proj.weight[ks],
                                               None if module.v_proj.bias is None else module.v_proj.bias[ks])
            q = module.q_norm(q.view(shape)).transpose(1, 2)
            k = module.k_norm(k.view(shape)).transpose(1, 2)
            v = v.view(shape).transpose(1, 2)
            q, k = _rope(q, k, *position_embeddings)
            kp, vp = pools[module.layer_idx]
            append_kv(kp, vp, k[:, :, 0, :], v[:, :, 0, :], targets, prepared.status,
                      tails if module.layer_idx == 0 else None)
            result = attention_matrix(q[:, :, 0, :].contiguous(), kp, vp, prepared)
            if decoder.world > 1:
                # rank-major concatenation along dim 0 (the form every backend accepts)
                gathered = torch.empty((decoder.world * nreq, decoder.local_hq, decoder.dim), device=result.device,
                                       dtype=result.dtype)
                torch.distributed.all_gather_into_tensor(gathered, result.contiguous(), group=decoder.group)
                result = gathered.view(decoder.world, nreq, decoder.local_hq, decoder.dim).permute(1, 0, 2, 3)
            return module.o_proj(result.reshape(nreq, 1, -1)), None

        return forward

    @torch.inference_mode()
    def step(self, token_ids):
        """Feed one token per request; returns next-token logits ``[NREQ, vocab]``."""
        token_ids = list(token_ids)
        if len(token_ids) != len(self.sequences):
            raise ValueError("one token per request")
        positions = torch.tensor([[len(s)] for s in self.sequences], device=self.device)
        targets = torch.tensor(self._append(token_ids), device=self.device)
        prepared = self._prepare_plan()
        forward = self._attention_forward(prepared, targets, len(token_ids))
        for layer in self.model.model.layers:
            layer.self_attn.forward = MethodType(forward, layer.self_attn)
        try:
            output = self.model(torch.tensor(token_ids, device=self.device)[:, None], position_ids=positions,
                                use_cache=False)
            self.logits = output.logits[:, 0]
        finally:
            for layer, original in zip(self.model.model.layers, self.original):
                layer.self_attn.forward = original
        return self.logits


class CachedPrefixDecoder(SharedKVDecoder):
    """Reuse the prompt schedule; only the tails' lengths change per step (reference qwen.py:106-124)."""

    def __init__(self, model, sequences, max_new_tokens=32, method="cube", cost_model=None, prefill="shared",
                 shard=None):
        super().__init__(model, sequences, max_new_tokens, method, cost_model, prefill, shard)
        prefix = schedule(self.tree, self.hq, self.hk, self.dim, self.method, self.cost_model)
        q = torch.empty((len(self.sequences), self.local_hq, self.dim), device=self.device, dtype=model.dtype)
        self.cached_plan = CachedDecodePlan(prefix, q, self.prefix_size, max_new_tokens, self.local_hk)

    def _append(self, token_ids):
        if self.generated >= self.max_new_tokens:
            raise ValueError("Decode exceeds allocated max_new_tokens")
        positions = self._next_positions(len(token_ids))
        for sequence, token in zip(self.sequences, token_ids):
            sequence.append(token)
        self.used += len(token_ids)
        return positions

    def _prepare_plan(self):
        return self.cached_plan.update(self.generated)

    @torch.inference_mode()
    def generate(self, steps, events=None):
        """Greedy decode of ``steps`` tokens per request, the whole step recorded once as a CUDA graph.

        One replay feeds every request the argmax of its previous logits
        (computed on the device), appends the new K/V rows at the tails, sets
        the tails' lengths in the plan on the device and runs the model: no
        host round trip between steps.  Afterwards ``sequences``, ``logits``,
        ``generated`` and ``used`` are as ``steps`` calls of
        ``step(logits.argmax(-1))`` leave them.  Returns the generated tokens
        ``[steps][NREQ]``.  ``events``, an optional (start, end) pair of
        ``torch.cuda.Event(enable_timing=True)``, is recorded around the
        replays alone (capture and warm-up excluded), for timing.
        """
        if steps <= 0:
            return []
        if self.generated + steps > self.max_new_tokens:
            raise ValueError("Decode exceeds allocated max_new_tokens")
        nreq, dev, t0 = len(self.sequences), self.device, self.generated
        t = torch.full((1,), t0, dtype=torch.int64, device=dev)            # tokens generated so far
        start_pos = torch.tensor([len(s) for s in self.sequences], dtype=torch.int64, device=dev)
        tail = torch.tensor([self.prefix_size + r * self.max_new_tokens for r in range(nreq)], dtype=torch.int64,
                            device=dev)
        first = self.logits.argmax(-1)
        tokens = first.clone()
        out = torch.zeros((steps, nreq), dtype=torch.int64, device=dev)
        positions = torch.empty((nreq, 1), dtype=torch.int64, device=dev)
        targets = torch.empty(nreq, dtype=torch.int64, device=dev)
        # the first layer's fused append sets the tails' lengths to t + 1
        forward = self._attention_forward(self.cached_plan.prepared, targets, nreq, (self.cached_plan, t, 1))

        def body():
            positions.copy_((start_pos + (t - t0))[:, None])
            targets.copy_(tail + t)
            out.index_copy_(0, (t - t0).clamp(max=steps - 1), tokens[None])
            # a prepared (empty) mask mapping: the patched attention needs no mask, and building one
            # would copy a host scalar, which a graph capture cannot record
            logits = self.model(tokens[:, None], position_ids=positions, use_cache=False,
                                attention_mask={"full_attention": None, "sliding_attention": None}).logits[:, 0]
            tokens.copy_(logits.argmax(-1))
            t.add_(1)
            return logits

        for layer in self.model.model.layers:
            layer.self_attn.forward = MethodType(forward, layer.self_attn)
        try:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                body()                                   # warm-up (lazy library setup); its writes are redone
            torch.cuda.current_stream(dev).wait_stream(side)
            t.fill_(t0)
            tokens.copy_(first)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                logits = body()
            if events is not None:
                events[0].record()
            for _ in range(steps):
                graph.replay()
            if events is not None:
                events[1].record()
            generated = out.tolist()
            self.logits = logits.clone()
            del graph
        finally:
            for layer, original in zip(self.model.model.layers, self.original):
                layer.self_attn.forward = original
        for row in generated:
            for sequence, token in zip(self.sequences, row):
                sequence.append(token)
        self.generated += steps
        self.used += steps * nreq
        return generated
