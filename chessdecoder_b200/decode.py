"""KV-cache inference backbone on the CUDA kernels: the counterpart of
chessdecoder/cpp/decoder/batched_backbone.{hpp,cpp} (``BatchedBackbone``),
which runs the exported module chessdecoder/export/backbone_causal.py
(``BackboneCausal.forward``: embedding with Fourier override, 12 pre-norm
layers with RoPE at explicit positions, attention over past + new keys under an
additive mask, SwiGLU MLP, final norm) through TorchScript with fp16 caches.

Here one batch of B sequences keeps two caches (causal and prefix, as the
reference), each preallocated in HBM:

* ``k`` / ``v``: bf16 [L, B, H, max_len, 64]; a step writes only its new rows;
* ``valid``: u8 [B, max_len], the reference's 0 / -1e9 mask buffer as one byte
  per key;
* ``len_dev``: the cache length as a device int32, read by the kernels, so a
  fixed-shape step replays from a CUDA graph; ``len`` is its host mirror.

Per layer a step runs RMSNorm -> fused q|k|v GEMM (fp32 out) -> ``kv_append``
(RoPE at the tokens' positions, q to a bf16 buffer, k / v into the cache) ->
``decode_attn`` -> output GEMM + residual -> RMSNorm -> SwiGLU GEMM -> down
GEMM + residual; then the final norm.  Weights are the training parameter
store's bf16 copies (the same ``state_dict`` layout as ChessDecoder).

The public methods mirror BatchedBackbone (batched_backbone.hpp:17-94) with the
same argument meaning: ids / pos [B, S] int64, override values [B, S] and mask
[B, S] bool (Fourier injection), active [B] bool, num_real [B] int64.  They
return the final-norm hidden state [B, S, E] (fp32; ``last_hidden16`` holds the
bf16 copy for the heads).  The incremental steps run from a CUDA graph after
their first call; their outputs are then the graph's static buffers, valid
until the next incremental step of the same cache.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch

from . import kernels as K
from .engine import ModelConfig, ParamStore, init_reference_weights, make_d_buckets, make_wl_buckets, rope_table

HEAD_DIM = 64


class KVCache:
    def __init__(self, L, B, H, max_len, device, name="cache"):
        self.name = name
        self.k = torch.zeros(L, B, H, max_len, HEAD_DIM, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        self.valid = torch.zeros(B, max_len, dtype=torch.uint8, device=device)
        self.len_dev = torch.zeros(1, dtype=torch.int32, device=device)
        self.len = 0

    def reset(self):
        """resetCausal / resetPrefix (batched_backbone.cpp:110-116, 184-190):
        empty cache, every key invalid.  Rows past ``len`` are rewritten before
        they are read, so k / v need no clearing."""
        self.valid.zero_()
        self.len_dev.zero_()
        self.len = 0


def _splits(M: int, N: int, K_: int, sms: int = 148) -> int:
    """K splits for a split-K projection of M rows x N output columns over K_
    inputs: about one wave of (128 x 256 tile, K slice) units, at least one
    64-deep k block each."""
    tiles = ((M + 127) // 128) * ((N + 255) // 256)
    return max(1, min(K_ // 64, sms // tiles))


def _u8(t, device):
    return None if t is None else t.to(device=device, dtype=torch.bool).contiguous().view(torch.uint8)


def _i64(t, device):
    return None if t is None else t.to(device=device, dtype=torch.int64).contiguous()


class BatchedBackbone:
    """Batched KV-cache backbone (dense ChessDecoder; the exported module has no
    MoE).  ``max_seq_len``: cache capacity (keys per sequence), default the
    model's."""

    def __init__(self, cfg: Optional[ModelConfig] = None, batch_size: int = 1, max_seq_len: Optional[int] = None,
                 state_dict=None, device="cuda", seed: int = 0, store: Optional[ParamStore] = None,
                 use_graphs: bool = True):
        cfg = cfg or ModelConfig()
        if cfg.moe_experts:
            raise ValueError("the KV-cache backbone covers the dense model")
        if cfg.head_dim != HEAD_DIM:
            raise ValueError(f"head_dim must be {HEAD_DIM}")
        self.cfg = cfg
        self.B = int(batch_size)
        self.max_len = int(max_seq_len or cfg.max_seq_len)
        self.device = torch.device(device)
        if store is None:
            store = ParamStore(dataclasses.replace(cfg, finetune=False), self.device, optimizer_state=False)
            sd = state_dict if state_dict is not None else init_reference_weights(cfg, seed)
            store.load_state_dict({k: v.to(self.device) for k, v in sd.items()})
        self.store = store
        self.rope = rope_table(max(cfg.max_seq_len, self.max_len), cfg.head_dim).to(self.device)
        L, H = cfg.num_layers, cfg.num_heads
        self.causal = KVCache(L, self.B, H, self.max_len, self.device, "causal")
        self.prefix = KVCache(L, self.B, H, self.max_len, self.device, "prefix")
        # incremental steps replay from CUDA graphs (first call eager, second captures)
        self.use_graphs = bool(use_graphs) and self.device.type == "cuda"
        self._graphs = {}
        self._gen = {}
        self._centers = {}
        st, E, F = store, cfg.embed_dim, cfg.ff
        self._layers = []
        for i in range(L):
            p = f"layers.{i}."
            self._layers.append(dict(
                wqkv=st.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight").view(3 * E, E),
                wo=st.bf16(p + "attn.output_proj.weight"), s1=st.param(p + "sa_norm.scale"),
                s2=st.param(p + "mlp_norm.scale"),
                w13=st.span(p + "mlp.w1.weight", p + "mlp.w3.weight").view(2 * F, E), w2=st.bf16(p + "mlp.w2.weight")))
        self._ar = {}
        self.last_hidden16 = None
        self._sms = (torch.cuda.get_device_properties(self.device).multi_processor_count
                     if self.device.type == "cuda" else 148)

    # -- lengths ------------------------------------------------------------
    @property
    def causal_len(self):
        return self.causal.len

    @property
    def prefix_len(self):
        return self.prefix.len

    def reset_causal(self):
        self.causal.reset()

    def reset_prefix(self):
        self.prefix.reset()

    # -- mask buffer helpers (batched_backbone.cpp:74-104) ------------------
    def mark_causal_valid(self, pos: int, active):
        K.decode_mark(self.causal.valid, self.B, self.causal.len_dev, start=int(pos), count=1,
                      active=_u8(active, self.device))

    def mark_prefix_valid(self, pos: int, active):
        K.decode_mark(self.prefix.valid, self.B, self.prefix.len_dev, start=int(pos), count=1,
                      active=_u8(active, self.device))

    def mark_causal_valid_range(self, start: int, count: int, active):
        K.decode_mark(self.causal.valid, self.B, self.causal.len_dev, start=int(start), count=int(count),
                      active=_u8(active, self.device))

    def mark_prefix_valid_range(self, start: int, count: int, active):
        K.decode_mark(self.prefix.valid, self.B, self.prefix.len_dev, start=int(start), count=int(count),
                      active=_u8(active, self.device))

    # -- core forward --------------------------------------------------------
    def _arange32(self, n):
        t = self._ar.get(n)
        if t is None:
            t = self._ar[n] = torch.arange(n, dtype=torch.int32, device=self.device)
        return t

    def _embed(self, ids, ov, om_u8):
        """tok_embedding, with the rows under the override mask replaced by the
        Fourier encoding of their value (backbone_causal.py:100-109: every row
        is encoded, then blended)."""
        cfg, st = self.cfg, self.store
        T, E, nf = ids.numel(), cfg.embed_dim, cfg.num_fourier_freq
        dev = self.device
        rows = self._arange32(T)
        ones = torch.ones(T, dtype=torch.uint8, device=dev)
        fvals = torch.empty(T, device=dev)
        feat = torch.empty(T, 2 * nf, device=dev)
        K.fourier_features(ov, ov, ones, torch.zeros_like(ones), None, None, st.param("fourier_encoder.frequencies"),
                           rows, fvals, feat)
        frows = torch.empty(T, E, device=dev)
        K.gemm_f32(feat, st.param("fourier_encoder.proj.weight"), frows, bias=st.param("fourier_encoder.proj.bias"),
                   M=T)
        slot = torch.empty(T, dtype=torch.int32, device=dev)
        K.decode_slots(om_u8, slot)
        h0 = torch.empty(T, E, device=dev)
        K.embed_fwd(ids, st.param("tok_embedding.weight"), slot, frows, h0)
        return h0

    def _forward(self, cache: KVCache, ids, pos, ov, om, *, block_mode, active=None, num_real=None, full=None):
        """One pass of S new tokens per sequence over ``cache`` (keys [0, len)
        plus the new block); writes the new k / v rows at [len, len + S) but
        leaves len and the validity bytes to the caller."""
        cfg, dev = self.cfg, self.device
        B, S = ids.shape
        if B != self.B:
            raise ValueError(f"batch {B} != {self.B}")
        if cache.len + S > self.max_len:
            raise ValueError(f"cache full: {cache.len} + {S} > {self.max_len}")
        E, F, H = cfg.embed_dim, cfg.ff, cfg.num_heads
        T = B * S
        ids = ids.to(device=dev, dtype=torch.int64).reshape(-1).contiguous()
        pos32 = pos.to(device=dev, dtype=torch.int32).reshape(-1).contiguous()
        ov = (torch.zeros(T, device=dev) if ov is None else
              ov.to(device=dev, dtype=torch.float32).reshape(-1).contiguous())
        om_u8 = (torch.zeros(T, dtype=torch.uint8, device=dev) if om is None else _u8(om, dev).reshape(-1))
        x = self._embed(ids, ov, om_u8)
        # A causal block into an empty cache with no padding is the training
        # forward's causal attention: q | k | v rows go through cdk_attn_fwd
        # (tensor cores) instead of the cache-attention kernel.
        fresh = (cache.len == 0 and block_mode == K.BLOCK_CAUSAL and full is None and S >= 16
                 and (num_real is None or bool((num_real == S).all())))
        if fresh:
            qkv16 = torch.empty(T, 3 * E, device=dev, dtype=torch.bfloat16)
            lse = torch.empty(B * H * S, device=dev)
        n1 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        qkv = torch.empty(T, 3 * E, device=dev)
        q16 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        ao = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        u = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
        h1 = torch.empty(T, E, device=dev)
        # Few rows (incremental steps, small blocks): 128 x 256 output tiles
        # would leave most SMs idle while the weights stream, so the
        # projections run split-K, reduce-adding fp32 partial sums into a zeroed
        # output (or into a copy of the residual); SwiGLU then runs on the sums.
        small = T <= 512
        if small:
            gu32 = torch.empty(T, 2 * F, device=dev)
        else:
            gu = torch.empty(T, 2 * F, device=dev, dtype=torch.bfloat16)
        for i, w in enumerate(self._layers):
            K.rmsnorm_fwd(x, w["s1"], y16=n1)
            if small:
                qkv.zero_()
                K.gemm(n1, w["wqkv"], kind=K.EPI_ATOMIC_F32, out=qkv, split_k=_splits(T, 3 * E, E, self._sms))
            else:
                K.gemm(n1, w["wqkv"], kind=K.EPI_STORE_F32, out=qkv)
            if fresh:
                K.kv_append(qkv, B, S, H, cache.k[i], cache.v[i], cache.len_dev, pos=pos32, rope=self.rope,
                            q_out=qkv16, qkv_out=True)
                K.attn_fwd(qkv16, ao, lse, B, B, S, H)
            else:
                K.kv_append(qkv, B, S, H, cache.k[i], cache.v[i], cache.len_dev, pos=pos32, rope=self.rope,
                            q_out=q16)
                K.decode_attn(q16, cache.k[i], cache.v[i], cache.len_dev, S, B, H, cache.valid, ao,
                              block_mode=block_mode, active=active, num_real=num_real, full_mask=full)
            xn = torch.empty(T, E, device=dev)
            if small:
                h1.copy_(x)
                K.gemm(ao, w["wo"], kind=K.EPI_ATOMIC_F32, out=h1, split_k=_splits(T, E, E, self._sms))
                K.rmsnorm_fwd(h1, w["s2"], y16=n1)
                gu32.zero_()
                K.gemm(n1, w["w13"], kind=K.EPI_ATOMIC_F32, out=gu32, split_k=_splits(T, 2 * F, E, self._sms))
                K.swiglu_f32(gu32, u)
                xn.copy_(h1)
                K.gemm(u, w["w2"], kind=K.EPI_ATOMIC_F32, out=xn, split_k=_splits(T, E, F, self._sms))
            else:
                K.gemm(ao, w["wo"], kind=K.EPI_RESID_F32, out=h1, resid=x)
                K.rmsnorm_fwd(h1, w["s2"], y16=n1)
                K.gemm(n1, w["w13"], kind=K.EPI_SWIGLU, out=u, out2=gu, half_n=F)
                K.gemm(u, w["w2"], kind=K.EPI_RESID_F32, out=xn, resid=h1)
            x = xn
        h16 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        h32 = torch.empty(T, E, device=dev)
        K.rmsnorm_fwd(x, self.store.param("norm.scale"), y16=h16, y32=h32)
        self.last_hidden16 = h16.view(B, S, E)
        return h32.view(B, S, E)

    # -- causal mode (batched_backbone.cpp:110-177) -------------------------
    def causal_forward(self, ids, pos, ov, om, active, num_real):
        """S new tokens, causal among the first num_real[b] of each sequence;
        those become valid keys and the cache grows by S."""
        B, S = ids.shape
        nr = _i64(num_real, self.device)
        h = self._forward(self.causal, ids, pos, ov, om, block_mode=K.BLOCK_CAUSAL, num_real=nr)
        K.decode_mark(self.causal.valid, B, self.causal.len_dev, start=-1, count=S, advance=S, num_real=nr)
        self.causal.len += S
        return h

    def causal_incremental(self, ids, pos, ov, om, active):
        """One token: its key is valid where active (marked first, as the
        reference does); the cache grows by 1."""
        return self._incremental(self.causal, ids, pos, ov, om, active)

    def causal_probe(self, ids, pos, ov, om):
        """S tokens over the valid cache and each other; no cache update."""
        return self._forward(self.causal, ids, pos, ov, om, block_mode=K.BLOCK_ALL)

    # -- prefix mode (batched_backbone.cpp:184-258) -------------------------
    def prefix_forward(self, ids, pos, mask, ov, om, active):
        """Full pass with an explicit additive mask [B, 1, S, len + S] (0 =
        attend); then keys [0, S) become valid where active, as the reference
        marks them."""
        B, S = ids.shape
        total = self.prefix.len + S
        m = mask.to(self.device)
        if m.dim() == 4:
            m = m[:, 0]
        if tuple(m.shape) != (B, S, total):
            raise ValueError(f"mask must be [B, 1, {S}, {total}]")
        full = (m > -1e4).to(torch.uint8).contiguous()
        act = _u8(active, self.device)
        h = self._forward(self.prefix, ids, pos, ov, om, block_mode=K.BLOCK_ALL, full=full)
        K.decode_mark(self.prefix.valid, B, self.prefix.len_dev, start=0, count=S, advance=S, active=act)
        self.prefix.len += S
        return h

    def prefix_incremental(self, ids, pos, ov, om, active):
        return self._incremental(self.prefix, ids, pos, ov, om, active)

    def prefix_block_forward(self, ids, pos, ov, om, active):
        """S tokens attending to the valid cache and, where active, to the
        whole block; the block's keys become valid where active."""
        B, S = ids.shape
        act = _u8(active, self.device)
        h = self._forward(self.prefix, ids, pos, ov, om, block_mode=K.BLOCK_ACTIVE, active=act)
        K.decode_mark(self.prefix.valid, B, self.prefix.len_dev, start=-1, count=S, advance=S, active=act)
        self.prefix.len += S
        return h

    def prefix_probe(self, ids, pos, ov, om):
        return self._forward(self.prefix, ids, pos, ov, om, block_mode=K.BLOCK_ALL)

    # -- greedy generation (causalBoardStep, torch_backbone.hpp:141-152) ---------
    def generate(self, ids, pos, n_steps: int, head: str = "board_head", lut=None, active=None,
                 temperature: float = 0.0, seed: int = 0, return_log_probs: bool = False):
        """Generation on the causal cache, entirely on the device: step k runs
        one incremental step, the `head` logits of its hidden state, picks a
        token (argmax at temperature <= 0, as causalBoardStep; otherwise a
        sample of softmax(logits / temperature), as sampleBatched, from a
        counter-based stream keyed by `seed`), maps it to the full vocabulary
        by `lut` (sub-vocabulary index -> token id; None = identity) and feeds
        it back as step k+1's input at position + 1.  The first step runs
        eagerly, the others replay one CUDA graph (no host synchronisation
        between steps).  ids / pos [B, 1]: the first input token and its
        position; active [B] (default all).  Returns the generated token ids
        [n_steps, B] (device), and with return_log_probs also their unscaled
        log-softmax values [n_steps, B] (the log-probabilities the reference
        records for GRPO)."""
        B = self.B
        cache = self.causal
        if n_steps <= 0:
            e = torch.empty(0, B, dtype=torch.int64, device=self.device)
            return (e, e.float()) if return_log_probs else e
        if cache.len + n_steps > self.max_len:
            raise ValueError(f"cache full: {cache.len} + {n_steps} > {self.max_len}")
        key = (head, None if lut is None else tuple(int(x) for x in lut), float(max(temperature, 0.0)))
        st = self._gen.get(key)
        if st is None:
            st = self._gen[key] = _GenState(self, head, lut, float(max(temperature, 0.0)))
        st.ids.copy_(ids.reshape(B, 1))
        st.pos.copy_(pos.reshape(B, 1))
        if active is None:
            st.active.fill_(True)
        else:
            st.active.copy_(active.reshape(B))
        st.seed.fill_(int(seed) & 0x7FFFFFFFFFFFFFFF)
        st.counter.zero_()
        self._gen_body(st)  # eager: every lazy set-up happens outside capture
        cache.len += 1
        if n_steps > 1 and not self.use_graphs:
            for _ in range(n_steps - 1):
                self._gen_body(st)
                cache.len += 1
        elif n_steps > 1:
            if st.graph is None:
                st.capture(self)
            for _ in range(n_steps - 1):
                st.graph.replay()
                K.LAUNCHES[0] += st.n_launch
                cache.len += 1
        out = st.hist[:n_steps].clone()
        return (out, st.lp_hist[:n_steps].clone()) if return_log_probs else out

    # -- value heads (evalWlHead / evalDHead, batched_engine.cpp:151-180) -------
    def value_head(self, name: str = "wl_head", h16=None, temperature: float = 0.0, seed: int = 0):
        """WL or D value head on hidden states h16 [B, E] bf16 (default: the
        last position of the latest call): Linear -> Mish -> Linear to bucket
        logits, a bucket picked as in cdk_head_select (argmax, or a sample at a
        temperature), its unscaled log-probability, and its centre value.
        Returns (bucket [B] int64, value [B] fp32, log_prob [B] fp32, logits)."""
        if name not in ("wl_head", "d_head"):
            raise ValueError("value heads are wl_head and d_head")
        st, cfg, dev = self.store, self.cfg, self.device
        if h16 is None:
            h16 = self.last_hidden16[:, -1, :]
        B = h16.shape[0]
        hv, nb = cfg.value_hidden_size, cfg.n_buckets
        z = torch.empty(B, hv, device=dev)
        K.gemm(h16, st.bf16(f"{name}.mlp.0.weight"), kind=K.EPI_STORE_F32, out=z, bias=st.param(f"{name}.mlp.0.bias"))
        a16 = torch.empty(B, hv, device=dev, dtype=torch.bfloat16)
        K.mish_bf16(z, a16)
        logits = torch.empty(B, nb, device=dev)
        K.gemm(a16, st.bf16(f"{name}.mlp.2.weight"), kind=K.EPI_STORE_F32, out=logits,
               bias=st.param(f"{name}.mlp.2.bias"))
        idx = torch.empty(B, dtype=torch.int64, device=dev)
        lp = torch.empty(B, device=dev)
        seed_t = torch.full((1,), int(seed) & 0x7FFFFFFFFFFFFFFF, dtype=torch.int64, device=dev)
        K.head_select(logits, idx, temperature=temperature, seed=seed_t, lp=lp)
        if name not in self._centers:
            self._centers[name] = (make_wl_buckets(cfg.n_buckets, cfg.wl_sigma) if name == "wl_head"
                                   else make_d_buckets(cfg.n_buckets)).to(dev)
        return idx, self._centers[name][idx], lp, logits

    def _gen_body(self, st):
        self._incremental_body(self.causal, st.ids, st.pos, None, None, st.active)
        K.gemm(self.last_hidden16.reshape(self.B, -1), st.weight, kind=K.EPI_STORE_F32, out=st.logits, bias=st.bias)
        K.head_select(st.logits, st.ids.view(-1), temperature=st.temperature, seed=st.seed, lut=st.lut,
                      pos=st.pos.view(-1), hist=st.hist, lp_hist=st.lp_hist, counter=st.counter)

    def _incremental(self, cache, ids, pos, ov, om, active):
        B, S = ids.shape
        if S != 1:
            raise ValueError("incremental steps take one token per sequence")
        if B != self.B:
            raise ValueError(f"batch {B} != {self.B}")
        if cache.len + 1 > self.max_len:
            raise ValueError(f"cache full: {cache.len} + 1 > {self.max_len}")
        g = self._graphs.get(cache.name) if self.use_graphs else None
        if g is None or g == "warm":
            if g == "warm":  # second call: capture, then replay below
                g = self._graphs[cache.name] = _IncrementalGraph(self, cache)
            else:
                if self.use_graphs:  # first call runs eagerly: every lazy set-up happens outside capture
                    self._graphs[cache.name] = "warm"
                h = self._incremental_body(cache, ids, pos, ov, om, active)
                cache.len += 1
                return h
        g.load(ids, pos, ov, om, active)
        g.graph.replay()
        K.LAUNCHES[0] += g.n_launch
        cache.len += 1
        self.last_hidden16 = g.out16
        return g.out

    def _incremental_body(self, cache, ids, pos, ov, om, active):
        B = ids.shape[0]
        act = _u8(active, self.device)
        K.decode_mark(cache.valid, B, cache.len_dev, start=-1, count=1, active=act)
        h = self._forward(cache, ids, pos, ov, om, block_mode=K.BLOCK_VALID)
        K.decode_mark(cache.valid, B, cache.len_dev, advance=1)
        return h


class _IncrementalGraph:
    """One incremental step of a cache captured as a CUDA graph: static input
    buffers, the whole 12-layer pass and the cache-length update replay as one
    launch.  The step reads the cache length on the device, so the same graph
    serves every position."""

    def __init__(self, bb: BatchedBackbone, cache: KVCache):
        dev, B = bb.device, bb.B
        self.ids = torch.zeros(B, 1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, 1, dtype=torch.int64, device=dev)
        self.ov = torch.zeros(B, 1, device=dev)
        self.om = torch.zeros(B, 1, dtype=torch.bool, device=dev)
        self.active = torch.ones(B, dtype=torch.bool, device=dev)
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(dev)
        n0 = K.LAUNCHES[0]
        with torch.cuda.graph(self.graph):
            self.out = bb._incremental_body(cache, self.ids, self.pos, self.ov, self.om, self.active)
        self.n_launch = K.LAUNCHES[0] - n0  # kernels of the library in one replay
        K.LAUNCHES[0] = n0
        self.out16 = bb.last_hidden16

    def load(self, ids, pos, ov, om, active):
        self.ids.copy_(ids.reshape(self.ids.shape), non_blocking=True)
        self.pos.copy_(pos.reshape(self.pos.shape), non_blocking=True)
        if ov is None:
            self.ov.zero_()
        else:
            self.ov.copy_(ov.reshape(self.ov.shape), non_blocking=True)
        if om is None:
            self.om.zero_()
        else:
            self.om.copy_(om.reshape(self.om.shape), non_blocking=True)
        if active is None:
            self.active.fill_(True)
        else:
            self.active.copy_(active.reshape(self.active.shape), non_blocking=True)


class _GenState:
    """Static buffers and the captured step of a greedy generation loop."""

    def __init__(self, bb: BatchedBackbone, head: str, lut, temperature: float = 0.0):
        dev, B = bb.device, bb.B
        self.temperature = temperature
        self.weight = bb.store.bf16(f"{head}.weight")
        self.bias = bb.store.param(f"{head}.bias")
        V = self.weight.shape[0]
        self.lut = None if lut is None else torch.as_tensor(list(lut), dtype=torch.int64, device=dev)
        if self.lut is not None and self.lut.numel() != V:
            raise ValueError(f"lut has {self.lut.numel()} entries, head {head} has {V} outputs")
        self.ids = torch.zeros(B, 1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, 1, dtype=torch.int64, device=dev)
        self.active = torch.ones(B, dtype=torch.bool, device=dev)
        self.logits = torch.empty(B, V, device=dev)
        self.hist = torch.zeros(bb.max_len, B, dtype=torch.int64, device=dev)
        self.lp_hist = torch.zeros(bb.max_len, B, device=dev)
        self.seed = torch.zeros(1, dtype=torch.int64, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph = None
        self.n_launch = 0

    def capture(self, bb: BatchedBackbone):
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(bb.device)
        n0 = K.LAUNCHES[0]
        with torch.cuda.graph(self.graph):
            bb._gen_body(self)
        self.n_launch = K.LAUNCHES[0] - n0
        K.LAUNCHES[0] = n0
