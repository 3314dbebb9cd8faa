"""One-token decode steps of several layers replayed from a CUDA graph.

A decode step of one layer is three small launches (append the new K/V rows, route, attend) whose
host-side preparation costs more than their GPU time at serving batch sizes.  ``DecodeStepGraph``
captures the launches of every layer of a step once, against static input / output buffers and a
device position vector, and replays them; the position vector is advanced inside the graph.  What
changes between steps on the host — a sequence completing its active chunk, whose summaries must be
built and (RAM tier) whose rows move into the window slots — runs eagerly after the replay, exactly
as ``ChunkRouter.decode_step`` defers it (chunk_router.py:631-657 closes after the block's
attention).

Requirements: one new token per sequence per step (L = 1), the stores' capacities already cover
every position the graph will reach (``capacity_tokens``), and the graph is replayed on the stream
it was captured for.  Results equal ``ChunkRouter.decode_step`` on the same inputs.
"""
from __future__ import annotations

from typing import List, Sequence

import torch

from . import ops
from .decode import _pool_size, close_chunk


class DecodeStepGraph:
    def __init__(self, router, layers: Sequence[int], seq_pos_host: List[int], capacity_tokens: int,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        cfg, store = router.cfg, router.store
        self.router, self.layers = router, list(layers)
        self.C = cfg.chunk_size
        self.capacity = int(capacity_tokens)
        B = len(seq_pos_host)
        dev = store.compute_device
        H, KVH, Dh = cfg.nhead, cfg.kv_heads, cfg.head_dim
        self.hp = cfg.hga_params(store.policy, B, dtype)
        ncap = (capacity_tokens + self.C - 1) // self.C
        for layer in self.layers:
            store.ensure_capacity(layer, ncap, ncap * self.C)
        self.pos_host = list(seq_pos_host)
        # the largest routed pool any replay can meet: Kc and Kg are fixed at capture, rows with
        # smaller pools pad their lists exactly as a mixed-length decode_step does
        self.nmid = max(1, _pool_size(store.policy, (capacity_tokens - 1) // self.C))
        if max(seq_pos_host) >= capacity_tokens:
            raise ValueError("seq_pos beyond capacity_tokens")
        self.seq_pos = torch.tensor(seq_pos_host, dtype=torch.int32, device=dev)
        n = len(self.layers)
        # one flat input vector per layer holding q [B,H,1,Dh] | k_rope | k_raw | v [B,KVH,1,Dh],
        # each segment contiguous: a caller fills a step with one copy per layer, and the kernels
        # read the segments in place
        nq, nk = B * H * Dh, B * KVH * Dh
        self.inputs = torch.zeros(n, nq + 3 * nk, device=dev, dtype=dtype)
        self.q = self.inputs[:, :nq].view(n, B, H, 1, Dh)
        self.k_rope = self.inputs[:, nq:nq + nk].view(n, B, KVH, 1, Dh)
        self.k_raw = self.inputs[:, nq + nk:nq + 2 * nk].view(n, B, KVH, 1, Dh)
        self.v = self.inputs[:, nq + 2 * nk:].view(n, B, KVH, 1, Dh)
        self.out = torch.zeros(n, B, H, 1, Dh, device=dev, dtype=dtype)
        self.graph = torch.cuda.CUDAGraph()
        self._capture()

    def _launch_all(self) -> None:
        store = self.router.store
        for i, layer in enumerate(self.layers):
            st = store.layer_buffers(layer)
            hot_k, hot_v = store.hot_buffers(layer)
            cold_k, cold_v = store.cold_buffers(layer)
            ops.append_tokens(self.hp, self.seq_pos, self.k_rope[i], self.v[i], self.k_raw[i], hot_k, hot_v,
                              store.hot_mode, None if store.hot_mode == 0 else cold_k,
                              None if store.hot_mode == 0 else cold_v, store.active_raw(layer))
            r = ops.route_decode(self.hp, self.q[i], self.seq_pos, st.chunk_k, st.group_k, self.nmid)
            ops.attend_decode(self.hp, self.q[i], self.seq_pos, hot_k, hot_v, store.hot_mode, cold_k, cold_v,
                              r["open_gid"], r["open_t0"], out=self.out[i])
        self.seq_pos.add_(1)

    def _capture(self) -> None:
        s = torch.cuda.Stream(self.seq_pos.device)
        s.wait_stream(torch.cuda.current_stream(self.seq_pos.device))
        # warm-up launch outside the graph (kernel attributes and tensor maps are set on first use);
        # its effects are undone by restoring the positions, and the appended rows are rewritten by
        # the first replay
        with torch.cuda.stream(s):
            saved = self.seq_pos.clone()
            self._launch_all()
            self.seq_pos.copy_(saved)
        torch.cuda.current_stream(self.seq_pos.device).wait_stream(s)
        torch.cuda.synchronize(self.seq_pos.device)
        with torch.cuda.graph(self.graph, stream=s):
            self._launch_all()

    def step(self) -> torch.Tensor:
        """Replay one step on the inputs already written into ``inputs`` [layers, flat] (or
        through its views ``q`` / ``k_rope`` / ``k_raw`` / ``v``, [layers, B, heads, 1, Dh]); returns ``out``
        [layers, B, H, 1, Dh] (overwritten by the next step).  Chunks completed by this step are
        closed afterwards, on the host's schedule."""
        C = self.C
        if max(self.pos_host) >= self.capacity:
            raise RuntimeError("DecodeStepGraph: a sequence reached capacity_tokens; build a larger graph")
        self.graph.replay()
        rows = [b for b, p in enumerate(self.pos_host) if p % C == C - 1]
        if rows:
            for layer in self.layers:
                close_chunk(self.router, layer, self.hp, [self.pos_host[b] // C for b in rows], rows=rows)
        self.pos_host = [p + 1 for p in self.pos_host]
        return self.out


__all__ = ["DecodeStepGraph"]
