"""Drop-in B200 replacements for the reference's fused SpecFold generators.

``SpecFoldTritonFastDLLMV2Generation`` (specfold/generate/fastdllm_v2_folded.py:226-370)
and ``SpecFoldTritonNLDGeneration`` (specfold/generate/nld_folded.py:244-394) override
one method, ``_batched_block_forward(batched_input [B1, N] int64, past_key_values) ->
logits [B1, N, V]``, the seam the Spiffy decoding loop calls
(fastdllm_v2_generation.py:634, nld_generation.py:247).  The classes here keep that
method, its helpers (``_build_parent_map``, ``_pack_layer_weights``, ``fold_ratio``,
``delta``, ``fold_bucket``) and their meaning, and run the layer loop as one call into
libspecfold_b200 (hand-written sm_100a kernels).  There is no Triton and no fallback to
a PyTorch or CPU path: a missing library or a device error raises.

Host-side work kept in Python, as in the reference: the parent map (one host sync),
the embedding lookup and RoPE tables (the model's own modules), and the fold counters
(a second small sync that also carries the device error word).

To use them inside the reference's decoding loop, mix ``FoldedVerifyB200`` in front of
the reference's base generator::

    class Gen(SpecFoldB200FastDLLMV2Generation, FastDLLMV2SpeculativeGeneration): ...

Standalone (tests, benchmarks) they need only ``model_executor.model``.
"""

from __future__ import annotations

import ctypes
import logging
from typing import Dict, List, Optional, Tuple

import torch

from . import _lib
from . import kernels as K
from .kernels import draft_blocks as K_draft_blocks
from .kernels import dtype_code

logger = logging.getLogger(__name__)


class FoldedVerifyB200:
    """Shared implementation; subclasses fix the model family."""

    family = "fastdllm"
    _packed_weights = None

    def __init__(self, *args, delta: float = 0.1, fold_bucket: Optional[int] = None, **kwargs):
        mro = type(self).__mro__
        if mro[mro.index(FoldedVerifyB200) + 1] is object:
            # standalone: only the executor is needed (positional or keyword)
            self.model_executor = kwargs.pop("model_executor", args[0] if args else None)
        else:
            # mixed in front of a reference generator: its __init__ takes the rest
            super().__init__(*args, **kwargs)
        self.delta = float(delta)
        # None: the compaction bucket is B1*N (every row fits); an int caps it
        # (fastdllm_v2_folded.py:230-235)
        self.fold_bucket = None if fold_bucket is None else int(fold_bucket)
        self._fold_stats: List[dict] = []
        self._ws: Dict[Tuple, torch.Tensor] = {}
        self.last_rec_masks: Optional[torch.Tensor] = None
        self.record_masks = False
        # True: the fold counters and the device error word of a call are read at the next
        # settle_stats() (or the next call with the same configuration) instead of a host
        # sync at the end of every call; used by decode loops, which synchronise anyway
        self.defer_stats = False
        # True: every call returns logits of its own (a copy of the library's output
        # buffer), which the decode loop may keep across calls -- it caches draft logits
        # for later hits (fastdllm_v2_generation.py:640-643).  False: the returned tensor
        # is the output buffer itself, valid until the next call with the same shapes.
        self.copy_logits = True

    # -------------------------------------------------------------- reference API
    @property
    def fold_ratio(self):
        """1 - recomputed / draft positions over all calls (fastdllm_v2_folded.py:49-53)."""
        tot = getattr(self, "_fold_draft_positions", 0)
        rec = getattr(self, "_fold_draft_recomputed", 0)
        return 1.0 - rec / tot if tot else float("nan")

    @staticmethod
    def _build_parent_map(batched_input: torch.Tensor) -> Tuple[List[Optional[int]], List[int]]:
        """par(i): the first branch whose differing-position set (vs the main block) is a
        one-smaller subset of draft i's, else main (0); one device->host sync
        (fastdllm_v2_folded.py:55-75)."""
        B1 = batched_input.shape[0]
        differs = batched_input != batched_input[0:1]
        escapes = (differs.unsqueeze(0) & ~differs.unsqueeze(1)).any(-1)
        both = torch.cat([differs.sum(1, dtype=torch.int64).unsqueeze(1),
                          escapes.to(torch.int64)], dim=1).tolist()
        counts = [row[0] for row in both]
        parent: List[Optional[int]] = [None] + [0] * (B1 - 1)
        for i in range(1, B1):
            for j in range(B1):
                if j != i and counts[j] == counts[i] - 1 and not both[i][1 + j]:
                    parent[i] = j
                    break
        return parent, counts

    def _base(self):
        m = self.model_executor.model
        return m.encoder if self.family == "nld" else m.model

    def _head(self):
        m = self.model_executor.model
        return m.diffusion_head if self.family == "nld" else m.lm_head

    # bf16 models: store every projection in the tile layout of the tensor-core GEMM
    # (one contiguous 16 KB read per pipeline stage); a one-time copy of the weights
    tile_weights = True

    @staticmethod
    def _tiles(w: torch.Tensor, w2: Optional[torch.Tensor] = None) -> torch.Tensor:
        lib = _lib.load()
        mode = 0 if w2 is None else 1
        n_out, K = w.shape
        inter = n_out if mode == 1 else 0
        out = torch.empty(lib.sf_weight_tiles_bytes(n_out * (2 if mode else 1), K, mode, inter)
                          // 2, dtype=w.dtype, device=w.device)
        _lib.check(lib.sf_pack_weight_tiles(w.data_ptr(), None if w2 is None else w2.data_ptr(),
                                            n_out, K, mode, inter, out.data_ptr(),
                                            torch.cuda.current_stream(w.device).cuda_stream),
                   "pack weight tiles")
        return out

    # -------------------------------------------------------------- tensor parallel
    # rank, size and the library's communicator of the 14B configuration; size 1 = off
    _tp = (0, 1, None)
    _tp_transport = None

    def set_tensor_parallel(self, rank: int, size: int, transport: Optional[str] = None,
                            max_rows: int = 256) -> None:
        """Shard every layer over `size` ranks (attention heads and the intermediate
        dimension); o_proj and down produce partial sums that are reduced across the ranks.
        Collective over the default torch.distributed group.

        transport "p2p" (default; SF_TP_TRANSPORT overrides): each rank's partials stay in
        an exchange buffer that every other rank maps through CUDA IPC, and the kernels
        consuming the sums read all ranks' partials over NVLink (sf_tp_peers_init).
        "nccl": the library's own NCCL communicator all-reduces them (sf_tp_comm_init;
        rank 0 creates the id and broadcasts it).  `max_rows` bounds B1 * N."""
        import os
        import torch.distributed as dist
        lib = _lib.load()
        self.close_tensor_parallel()
        if size <= 1:
            return
        transport = transport or os.environ.get("SF_TP_TRANSPORT", "p2p")
        self._tp_transport = transport
        if transport == "nccl":
            uid = (ctypes.c_char * 128)()
            if rank == 0:
                _lib.check(lib.sf_tp_unique_id(ctypes.cast(uid, ctypes.c_void_p), 128), "tp id")
            box = [bytes(uid) if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            ctypes.memmove(uid, box[0], 128)
            comm = ctypes.c_void_p()
            _lib.check(lib.sf_tp_comm_init(ctypes.cast(uid, ctypes.c_void_p), size, rank,
                                           ctypes.byref(comm)), "tp communicator")
            self._tp = (rank, size, comm.value)
        elif transport == "p2p":
            D = self.model_executor.model.config.hidden_size
            dev = torch.device("cuda", torch.cuda.current_device())
            nbytes = lib.sf_tp_exchange_bytes(max_rows, D)
            xbuf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
            torch.cuda.synchronize(dev)
            h = (ctypes.c_char * 64)()
            off = ctypes.c_size_t()
            _lib.check(lib.sf_tp_ipc_export(xbuf.data_ptr(), ctypes.cast(h, ctypes.c_void_p), 64,
                                            ctypes.byref(off)), "tp ipc export")
            handles = [None] * size
            dist.all_gather_object(handles, (bytes(h), off.value))
            # each peer's buffer mapped into THIS device's context (the kernels reading it
            # run here)
            mapped, ptrs = [], []
            for q in range(size):
                if q == rank:
                    ptrs.append(xbuf.data_ptr())
                    continue
                hq = (ctypes.c_char * 64).from_buffer_copy(handles[q][0])
                base = ctypes.c_void_p()
                _lib.check(lib.sf_tp_ipc_open(ctypes.cast(hq, ctypes.c_void_p), 64,
                                              ctypes.byref(base)), "tp ipc open")
                mapped.append(base.value)
                ptrs.append(base.value + handles[q][1])
            peers = ctypes.c_void_p()
            _lib.check(lib.sf_tp_peers_init(rank, size, (ctypes.c_void_p * size)(*ptrs), max_rows,
                                            D, ctypes.byref(peers)), "tp peer table")
            self._tp_xbuf = (xbuf, mapped)
            self._tp_peers = peers.value
            self._tp = (rank, size, None)
            dist.barrier()          # every rank's buffer is mapped before any forward runs
        else:
            raise ValueError(f"tensor-parallel transport {transport!r}")
        self._packed_weights = None
        self.__dict__.pop("_statics", None)

    def close_tensor_parallel(self) -> None:
        """Release the captured graphs (they hold the collective calls), then the
        communicator or the peer table."""
        lib = _lib.load()
        lib.sf_release_graphs()
        self.__dict__.pop("_statics", None)
        if self._tp[2] is not None:
            _lib.check(lib.sf_tp_comm_destroy(self._tp[2]), "tp communicator")
        if getattr(self, "_tp_peers", None):
            _lib.check(lib.sf_tp_peers_destroy(self._tp_peers), "tp peer table")
            self._tp_peers = None
            xbuf, mapped = self._tp_xbuf
            torch.cuda.synchronize()
            for base in mapped:
                _lib.check(lib.sf_tp_ipc_close(base), "tp ipc close")
            self._tp_xbuf = None
        self._tp = (0, 1, None)

    @staticmethod
    def tp_shard(q_w, k_w, v_w, q_b, k_b, v_b, o_w, g_w, u_w, d_w, heads, kv_heads, rank, size):
        """This rank's shard of one layer: q heads [r*H/s, (r+1)*H/s) with their kv heads
        (GQA groups stay whole), o_proj's matching input columns, and rows / columns
        [r*I/s, (r+1)*I/s) of gate+up / down.  Returns (w_qkv, b_qkv, w_o, w_g, w_u, w_d)."""
        hd = q_w.shape[0] // heads
        if heads % size or kv_heads % size or g_w.shape[0] % size:
            raise ValueError(f"heads {heads} / kv heads {kv_heads} / intermediate "
                             f"{g_w.shape[0]} not divisible by {size} ranks")
        hq, hk, inter = heads // size, kv_heads // size, g_w.shape[0] // size
        qs = slice(rank * hq * hd, (rank + 1) * hq * hd)
        ks = slice(rank * hk * hd, (rank + 1) * hk * hd)
        isl = slice(rank * inter, (rank + 1) * inter)
        w_qkv = torch.cat([q_w[qs], k_w[ks], v_w[ks]], 0).contiguous()
        b_qkv = None if q_b is None else torch.cat([q_b[qs], k_b[ks], v_b[ks]], 0).contiguous()
        return (w_qkv, b_qkv, o_w[:, qs].contiguous(), g_w[isl].contiguous(),
                u_w[isl].contiguous(), d_w[:, isl].contiguous())

    def _pack_layer_weights(self, layers) -> None:
        """Per layer: [Wq; Wk; Wv] and its bias packed once (one weight stream for the
        QKV projection, fastdllm_v2_folded.py:77-87).  For bf16 models every projection is
        also laid out in 128x64 tiles for the tensor-core GEMM, gate and up interleaved
        per tile (the reference's [Wg; Wu] packing, done tile by tile).  Under tensor
        parallelism each rank packs its shard (tp_shard)."""
        packed = []
        tp_rank, tp_size, _ = self._tp
        cfg = self.model_executor.model.config
        for lyr in layers:
            a, mlp = lyr.self_attn, lyr.mlp
            if tp_size > 1:
                bq = a.q_proj.bias
                w_qkv, b_qkv, w_o, w_g, w_u, w_d = self.tp_shard(
                    a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, bq,
                    None if bq is None else a.k_proj.bias, None if bq is None else a.v_proj.bias,
                    a.o_proj.weight, mlp.gate_proj.weight, mlp.up_proj.weight,
                    mlp.down_proj.weight, cfg.num_attention_heads, cfg.num_key_value_heads,
                    tp_rank, tp_size)
            else:
                w_qkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous()
                if a.q_proj.bias is not None:
                    b_qkv = torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias], 0).contiguous()
                else:
                    b_qkv = None   # NLD: no bias (nld_folded.py:92-102 packs zeros)
                w_o = a.o_proj.weight.contiguous()
                w_g, w_u = mlp.gate_proj.weight.contiguous(), mlp.up_proj.weight.contiguous()
                w_d = mlp.down_proj.weight.contiguous()
            if self._use_tiles(w_qkv):
                w_qkv, w_o, w_g, w_u, w_d = (self._tiles(w_qkv), self._tiles(w_o),
                                             self._tiles(w_g, w_u), None, self._tiles(w_d))
            ws = (w_qkv, b_qkv, lyr.input_layernorm.weight.contiguous(), w_o,
                  lyr.post_attention_layernorm.weight.contiguous(), w_g, w_u, w_d)
            packed.append(ws)
        self._packed_weights = packed
        head_w = self._head().weight.contiguous()
        self._lm_w = self._tiles(head_w) if self._use_tiles(head_w) else head_w
        self._tiled = self._use_tiles(head_w)

    def _use_tiles(self, w: torch.Tensor) -> bool:
        return bool(self.tile_weights) and w.dtype == torch.bfloat16 and w.is_cuda

    def _shift_logits(self, logits: torch.Tensor) -> torch.Tensor:
        return torch.cat([logits[:, :1, :], logits[:, :-1, :]], dim=1)

    # -------------------------------------------------------------- the seam
    @torch.no_grad()
    def _batched_block_forward(self, batched_input: torch.Tensor, past_key_values) -> torch.Tensor:
        B1, N = batched_input.shape
        bucket = B1 * N if self.fold_bucket is None else max(1, min(self.fold_bucket, B1 * N))
        logits, stats = self._run(batched_input, past_key_values, bucket)
        if stats["max_count"] is not None and stats["max_count"] > bucket:
            # the reference re-runs its PyTorch path on overflow (fastdllm_v2_folded.py:367-369);
            # here the same kernels run again with room for every row
            logger.warning("SpecFold bucket overflow (%d > %d); re-running with bucket %d",
                           stats["max_count"], bucket, B1 * N)
            logits, stats = self._run(batched_input, past_key_values, B1 * N, count_stats=False)
        return logits

    def _workspace(self, key, nbytes, device) -> torch.Tensor:
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    @torch.no_grad()
    def dense_block_forward(self, batched_input: torch.Tensor, past_key_values) -> torch.Tensor:
        """The base generators' dense batched block forward -- every branch computed in
        full against the shared prefix (fastdllm_v2_generation.py:151-186,
        nld_generation.py:77-105) -- on the same kernels: with a negative threshold the
        gate recomputes every row, and the folded forward is then the dense one
        (fastdllm_v2_folded.py:6).  Used for the vanilla / unfolded comparisons; the fold
        counters are left alone.  Returns logits [B1, N, V] (shifted for Fast-dLLM)."""
        B1, N = batched_input.shape
        logits, _ = self._run(batched_input, past_key_values, B1 * N, count_stats=False, delta=-1.0)
        return logits

    @torch.no_grad()
    def commit_block_forward(self, block: torch.Tensor, cache, logits: bool = True):
        """The block commit forward of the decoding loops on the same kernels: the dense
        forward of one block [1, N] against the running prefix with every layer's keys
        and values of the block appended to ``cache`` (a PreallocatedKVCache) at
        positions [P, P + N) -- the executor call with update_past_key_values=True
        (fastdllm_v2_generation.py:562-568; nld_generation.py:283-289), which the
        reference runs as the model's dense forward plus DynamicCache.update.  Returns
        the model's unshifted logits [1, N, V] (the loop reads the last position's), or
        None with ``logits=False``, which skips the final norm and the LM head (the prompt
        blocks of a prefill)."""
        from .kv_cache import PreallocatedKVCache
        if not isinstance(cache, PreallocatedKVCache):
            raise TypeError("the commit forward appends to a PreallocatedKVCache")
        if block.dim() != 2 or block.shape[0] != 1:
            raise ValueError(f"the commit forward takes one block [1, N], got {tuple(block.shape)}")
        N = block.shape[1]
        cache.reserve(N)
        out, _ = self._run(block, cache, N, count_stats=False, delta=-1.0, commit=True,
                           shift=False, want_logits=logits)
        cache.advance(N)
        return out

    @torch.no_grad()
    def prefill_forward(self, tokens: torch.Tensor, cache, block: int = 32, logits: bool = True,
                        max_blocks: int = 16):
        """Commit a prompt of k * block tokens ([1, T] or [T]) to a PreallocatedKVCache in
        block-causal forwards of up to ``max_blocks`` blocks each (sf_verify_args.prefill):
        the same result as committing the blocks one at a time -- each block attends to
        the prefix, to the earlier blocks and to itself bidirectionally -- with the weights
        streamed once per chunk instead of once per block.  Returns the unshifted logits
        [1, block, V] of the last block (the executor's next-token row), or None."""
        from .kv_cache import PreallocatedKVCache
        if not isinstance(cache, PreallocatedKVCache):
            raise TypeError("the prefill forward appends to a PreallocatedKVCache")
        ids = tokens.reshape(-1)
        T = ids.numel()
        if T == 0 or T % block:
            raise ValueError(f"prefill of {T} tokens: a positive multiple of {block} expected")
        out = None
        for s0 in range(0, T, block * max_blocks):
            chunk = ids[s0:s0 + block * max_blocks]
            k = chunk.numel() // block
            last = s0 + chunk.numel() >= T
            cache.reserve(k * block)
            if k == 1:
                out, _ = self._run(chunk.view(1, block), cache, block, count_stats=False,
                                   delta=-1.0, commit=True, shift=False,
                                   want_logits=logits and last)
            else:
                out, _ = self._run(chunk.view(k, block), cache, k * block, count_stats=False,
                                   delta=-1.0, commit=True, shift=False,
                                   want_logits=logits and last, prefill=True)
            cache.advance(k * block)
        return out

    def _run(self, batched_input, past_key_values, bucket, count_stats=True, delta=None,
             commit=False, shift=None, want_logits=True, prefill=False):
        lib = _lib.load()
        m_ = self.model_executor.model
        base = self._base()
        cfg = m_.config
        dev = batched_input.device
        if dev.type != "cuda":
            raise ValueError("the B200 folded forward runs on CUDA tensors only")
        B1, N = batched_input.shape
        BN = B1 * N
        if self._packed_weights is None:
            self._pack_layer_weights(base.layers)
        P = int(past_key_values.get_seq_length()) if past_key_values is not None else 0
        stream = torch.cuda.current_stream(dev)
        emb = base.embed_tokens
        table = isinstance(emb, torch.nn.Embedding) and emb.max_norm is None
        hidden = None if table else emb(batched_input)
        dtype = emb.weight.dtype if table else hidden.dtype
        shift = (self.family == "fastdllm") if shift is None else bool(shift)
        st = self._static_state(batched_input, past_key_values, dtype, P, bucket,
                                commit=commit, shift=shift, want_logits=want_logits,
                                prefill=prefill)
        L = st["L"]
        if st["P_dev"] is not None:
            # one state (and captured graph) for every prefix length of the cache: the
            # length and its RoPE rows go to the device, the launches stay the same
            nr = B1 * N if prefill else N          # rows with their own positions
            if P + nr > st["cap"]:
                raise ValueError(f"prefix {P} + {nr} rows exceeds the cache capacity {st['cap']}")
            st["P_dev"].fill_(P)
            st["cos"].copy_(st["cos_all"][P:P + nr])
            st["sin"].copy_(st["sin_all"][P:P + nr])
            if st["q_scale"] is not None:
                st["q_scale"].copy_(st["q_scale_all"][P:P + nr])

        # per call: parent map on the device (the reference's :263-265 host round trip),
        # embeddings into the fixed input buffer, then the forward (a CUDA graph replay
        # once the argument set has been seen)
        ids = batched_input if batched_input.dtype == torch.int64 else batched_input.to(torch.int64)
        ids = ids.contiguous()
        _lib.check(lib.sf_parent_map(ids.data_ptr(), B1, N, st["par"].data_ptr(),
                                     stream.cuda_stream), "parent map")
        if table:   # the embedding lookup written straight into the fixed input buffer
            torch.index_select(emb.weight, 0, ids.view(-1), out=st["hidden"])
        else:
            st["hidden"].copy_(hidden.reshape(BN, -1))
        st["args"].stream = stream.cuda_stream
        st["args"].delta = self.delta if delta is None else float(delta)
        _lib.check(lib.sf_folded_verify_forward(st["args"]), "folded verify forward")
        logits = st["logits"]
        if logits is not None and self.copy_logits:
            logits = logits.clone()
        rec = st["rec"].clone() if st["rec"] is not None else None

        if rec is not None:
            self.last_rec_masks = rec.view(L, B1, N)
        host = st["host_slab"]
        if self.defer_stats and bucket >= BN:
            # decode loops: no overflow is possible (every row fits the bucket), so the fold
            # counters and the error word are read at the caller's next synchronisation
            # (settle_stats) instead of a sync of their own per call
            self._settle(st)
            host.copy_(st["slab"], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            st["pending"] = (ev, count_stats, B1, N, L)
            return logits, {"max_count": None, "sum_count": None}
        # one sync for the fold counters and the device error word (the reference's :363)
        host.copy_(st["slab"], non_blocking=True)
        stream.synchronize()
        counts = host[:L].tolist()
        bits = int(host[-1])
        if bits:
            raise _lib.SpecFoldError("folded verify forward: " + _lib.describe_device_error(bits))
        mx, sm = max(counts), sum(counts)
        if count_stats:
            self._count_folds(B1, N, L, sm)
        return logits, {"max_count": int(mx), "sum_count": int(sm)}

    def _count_folds(self, B1, N, L, recomputed_rows):
        self._fold_draft_positions = getattr(self, "_fold_draft_positions", 0) + (B1 - 1) * N * L
        self._fold_draft_recomputed = (getattr(self, "_fold_draft_recomputed", 0)
                                       + int(recomputed_rows) - L * N)

    def _settle(self, st) -> None:
        pend = st.get("pending")
        if pend is None:
            return
        st["pending"] = None
        ev, count_stats, B1, N, L = pend
        ev.synchronize()
        host = st["host_slab"]
        bits = int(host[-1])
        if bits:
            raise _lib.SpecFoldError("folded verify forward: " + _lib.describe_device_error(bits))
        if count_stats:
            self._count_folds(B1, N, L, sum(host[:L].tolist()))

    def settle_stats(self) -> None:
        """Read the fold counters and device error words of calls made with
        ``defer_stats`` (waits for them); raises SpecFoldError on a device error."""
        for st in list(self.__dict__.get("_statics", {}).values()):
            self._settle(st)

    def _static_state(self, batched_input, past_key_values, dtype, P, bucket, commit=False,
                      shift=True, want_logits=True, prefill=False) -> dict:
        """Buffers and the C argument struct of one configuration (shape, prefix cache
        tensors, bucket), kept at fixed addresses across calls so that the library
        replays its CUDA graph of the forward.  RoPE tables and the query scale depend
        only on the prefix length and are filled once here.

        With a PreallocatedKVCache the prefix length is not part of the configuration:
        it is handed to the kernels in device memory (sf_verify_args.P_dev), bounded by
        the cache capacity, and the RoPE rows of the current positions are copied from
        tables over the whole capacity at each call, so one state and one captured graph
        serve every block of a decode."""
        from .kv_cache import PreallocatedKVCache
        prealloc = isinstance(past_key_values, PreallocatedKVCache)
        lib = _lib.load()
        base = self._base()
        cfg = self.model_executor.model.config
        dev = batched_input.device
        layers = base.layers
        L = len(layers)
        B1, N = batched_input.shape
        BN = B1 * N
        tp_rank, tp_size, tp_comm = self._tp
        H, Hkv = cfg.num_attention_heads // tp_size, cfg.num_key_value_heads // tp_size
        hd = layers[0].self_attn.head_dim
        kv, keep, kv_stride = [], [], 0
        statics = self.__dict__.setdefault("_statics", {})
        if prealloc:
            # the cache's whole buffers (capacity rows per head): their addresses do not
            # change with the prefix length, and the store's address stands for all of
            # them (looked up first: a decode step skips the per-layer walk)
            fast = (dev.index, dtype, B1, N, "store", past_key_values._store.data_ptr(),
                    past_key_values.capacity, bucket, bool(self.record_masks), tp_size, tp_comm,
                    getattr(self, "_tp_peers", None), bool(commit), bool(shift),
                    bool(want_logits), bool(prefill))
            st = statics.get(fast)
            if st is not None:
                return st
            for li in range(L):
                k0, v0 = past_key_values.buffers(li)
                if tp_size > 1 and k0.shape[0] == Hkv * tp_size:   # this rank's kv heads
                    k0, v0 = k0[tp_rank * Hkv:(tp_rank + 1) * Hkv], v0[tp_rank * Hkv:(tp_rank + 1) * Hkv]
                keep += [k0, v0]
                kv.append((k0.data_ptr(), v0.data_ptr()))
            kv_stride = keep[0].stride(0)
            cap = past_key_values.capacity
        elif P > 0:
            for li in range(L):
                k, v = past_key_values[li]
                k0, v0 = self._prefix_view(k), self._prefix_view(v)
                if tp_size > 1 and k0.shape[0] == Hkv * tp_size:   # this rank's kv heads
                    k0, v0 = k0[tp_rank * Hkv:(tp_rank + 1) * Hkv], v0[tp_rank * Hkv:(tp_rank + 1) * Hkv]
                if kv_stride == 0:
                    kv_stride = k0.stride(0)
                if k0.stride(0) != kv_stride or v0.stride(0) != kv_stride:
                    raise ValueError("prefix cache layers must share one head stride")
                keep += [k0, v0]
                kv.append((k0.data_ptr(), v0.data_ptr()))
        if prealloc:
            key = fast
        else:
            key = (dev.index, dtype, B1, N, P, bucket, bool(self.record_masks), kv_stride,
                   tuple(kv), tp_size, tp_comm, getattr(self, "_tp_peers", None), bool(commit),
                   bool(shift), bool(want_logits))
            st = statics.get(key)
            if st is not None:
                return st

        D = layers[0].self_attn.q_proj.weight.shape[1]
        I = layers[0].mlp.gate_proj.weight.shape[0] // tp_size
        V = self._head().weight.shape[0]
        scale = float(layers[0].self_attn.scaling)
        nr = BN if prefill else N                    # rows with their own RoPE position
        probe = torch.zeros(1, nr, D, dtype=dtype, device=dev)
        pos = torch.arange(P, P + nr, device=dev).unsqueeze(0)
        cos, sin = base.rotary_emb(probe, pos)
        st = {"L": L, "keep": keep, "P_dev": None, "pending": None}
        st["cos"] = cos[0].to(dtype).contiguous()
        st["sin"] = sin[0].to(dtype).contiguous()
        st["q_scale"] = self._q_scale(cfg, P, nr, dev)
        P_bound = P
        if prealloc:
            P_bound = cap - nr
            st["cap"] = cap
            st["P_dev"] = torch.full((1,), P, dtype=torch.int32, device=dev)
            probe_all = torch.zeros(1, cap, D, dtype=dtype, device=dev)
            cos_all, sin_all = base.rotary_emb(probe_all, torch.arange(cap, device=dev).unsqueeze(0))
            st["cos_all"] = cos_all[0].to(dtype).contiguous()
            st["sin_all"] = sin_all[0].to(dtype).contiguous()
            qs_all = self._q_scale(cfg, 0, cap, dev, force=True)
            st["q_scale_all"] = qs_all
            st["q_scale"] = None if qs_all is None else qs_all[P:P + nr].clone()
        st["hidden"] = torch.empty(BN, D, dtype=dtype, device=dev)
        st["par"] = torch.zeros(B1, dtype=torch.int64, device=dev)
        st["logits"] = (torch.empty(1 if prefill else B1, N, V, dtype=dtype, device=dev)
                        if want_logits else None)
        st["slab"] = torch.zeros(L + L * B1 + 1, dtype=torch.int32, device=dev)
        st["host_slab"] = torch.zeros(L + L * B1 + 1, dtype=torch.int32).pin_memory()
        st["rec"] = torch.zeros(L * BN, dtype=torch.int8, device=dev) if self.record_masks else None
        need = lib.sf_verify_workspace_bytes(dtype_code(st["hidden"]), B1, N, D, H, Hkv, hd, I, V,
                                             P_bound + (BN if prefill else 0))
        st["ws"] = torch.empty(need, dtype=torch.uint8, device=dev)

        layer_arr = (_lib.SfLayer * L)()
        for li in range(L):
            w = self._packed_weights[li]
            sl = layer_arr[li]
            sl.w_qkv, sl.ln1_w, sl.w_o, sl.ln2_w = (w[0].data_ptr(), w[2].data_ptr(),
                                                    w[3].data_ptr(), w[4].data_ptr())
            sl.b_qkv = None if w[1] is None else w[1].data_ptr()
            sl.w_gate, sl.w_down = w[5].data_ptr(), w[7].data_ptr()
            sl.w_up = None if w[6] is None else w[6].data_ptr()
            if kv:
                sl.prefix_k, sl.prefix_v = kv[li]
        slab = st["slab"]
        args = _lib.SfVerifyArgs()
        args.dtype = dtype_code(st["hidden"])
        args.B1, args.N, args.D, args.H, args.Hkv, args.hd = B1, N, D, H, Hkv, hd
        args.I, args.V, args.L, args.P = I, V, L, P_bound
        args.kv_head_stride = kv_stride
        args.P_dev = None if st["P_dev"] is None else st["P_dev"].data_ptr()
        args.commit = 1 if commit else 0
        args.prefill = 1 if prefill else 0
        args.bucket = bucket
        args.delta = self.delta
        args.eps = float(getattr(cfg, "rms_norm_eps", 1e-6))
        args.scale = scale
        args.shift_logits = 1 if shift else 0
        args.weights_tiled = 1 if self._tiled else 0
        args.layers = layer_arr
        args.final_norm_w = base.norm.weight.data_ptr()
        args.lm_w = self._lm_w.data_ptr()
        args.par_idx = st["par"].data_ptr()
        args.hidden_in = st["hidden"].data_ptr()
        args.cos, args.sin = st["cos"].data_ptr(), st["sin"].data_ptr()
        args.q_scale = None if st["q_scale"] is None else st["q_scale"].data_ptr()
        args.logits = None if st["logits"] is None else st["logits"].data_ptr()
        args.count_slab = slab[:L].data_ptr()
        args.segcnt_slab = slab[L:L + L * B1].data_ptr()
        args.rec_slab = None if st["rec"] is None else st["rec"].data_ptr()
        args.ws = st["ws"].data_ptr()
        args.ws_bytes = st["ws"].numel()
        args.err = slab[L + L * B1:].data_ptr()
        args.tp_comm = tp_comm
        args.tp_size = tp_size
        args.tp_peers = getattr(self, "_tp_peers", None) if tp_size > 1 else None
        st["layer_arr"] = layer_arr
        st["args"] = args
        if len(statics) >= 12:      # a decode keeps one state per branch count + the commit
            self._settle(statics.pop(next(iter(statics))))
        statics[key] = st
        return st

    @staticmethod
    def _prefix_view(t: torch.Tensor) -> torch.Tensor:
        """[1, Hkv, P, hd] cache tensor -> [Hkv, P, hd] view with contiguous rows."""
        t0 = t[0]
        if t0.stride(2) != 1 or t0.stride(1) != t0.shape[2]:
            t0 = t0.contiguous()
        return t0

    def _q_scale(self, cfg, P, N, device, force=False):
        return None

    # -------------------------------------------------------------- draft construction
    def _graph_pairs(self, device):
        """The calibration graph's nodes with a non-empty ij_set and their (pos_rank,
        vocab_rank) pairs as device tensors, cached per graph object."""
        graph = getattr(self, "calibration_graph", None)
        if graph is None:
            return None
        key = (id(graph), str(device))
        cache = self.__dict__.setdefault("_graph_pairs_cache", {})
        hit = cache.get(key)
        if hit is not None and hit[0] is graph:
            return hit[1]
        nodes = [n for n in graph.get("selected_nodes", []) if n.get("ij_set")]
        pairs, off = [], [0]
        for n in nodes:
            pairs += [(int(i), int(j)) for i, j in n["ij_set"]]
            off.append(len(pairs))
        K = 1 + max((j for _, j in pairs), default=0)
        out = (nodes,
               torch.tensor(pairs or [(0, 0)], dtype=torch.int32, device=device).reshape(-1, 2),
               torch.tensor(off, dtype=torch.int32, device=device), K)
        cache[key] = (graph, out)
        return out

    def _draft_states_async(self, block, logits, mask, pos_offset, conf_fp32=False):
        """(nodes, drafts [n_nodes, L], valid [n_nodes]) from sf_draft_blocks, left on the
        device (no host sync); nodes == [] when the graph has no usable node."""
        g = self._graph_pairs(block.device)
        if g is None or not g[0]:
            return [], None, None
        nodes, pairs, off, K = g
        drafts, valid = K_draft_blocks(logits, mask, block, pos_offset, pairs, off, K, conf_fp32)
        return nodes, drafts, valid

    def _draft_states(self, block, logits, mask, pos_offset, conf_fp32):
        """(nodes, drafts [n_nodes, L], valid list) from sf_draft_blocks; one host sync."""
        g = self._graph_pairs(block.device)
        if g is None or not g[0]:
            return [], None, []
        nodes, pairs, off, K = g
        drafts, valid = K_draft_blocks(logits, mask, block, pos_offset, pairs, off, K, conf_fp32)
        return nodes, drafts, valid.tolist()


class SpecFoldB200FastDLLMV2Generation(FoldedVerifyB200):
    """Fast-dLLM v2 (Qwen2 backbone): QKV bias, shifted logits
    (replaces SpecFoldTritonFastDLLMV2Generation)."""

    family = "fastdllm"

    def _sample_with_top_p(self, logits: torch.Tensor, top_p: float = 0.95,
                           temperature: float = 0.0):
        """The decode loops' sampler (fastdllm_v2_generation.py:134-149 ->
        FastDLLMModelExecutor.sample_with_top_p) on the GPU for greedy decoding: tokens
        and their top-p filtered probabilities without sorting the vocabulary
        (sf_sample_top_p_greedy).  The probabilities come back as the tokens'
        confidence broadcast over the vocabulary dimension (a stride-0 view of shape
        logits.shape): the loops only gather them at the sampled token (:348-351) and
        slice positions (:615-616).  There is no fallback to the reference's sampler:
        temperature sampling, CPU logits and other dtypes raise NotImplementedError."""
        if temperature > 0 or not logits.is_cuda or logits.dtype not in (torch.bfloat16, torch.float32):
            raise NotImplementedError("the GPU sampler is greedy (temperature 0) on CUDA bf16 / "
                                      f"fp32 logits (got temperature {temperature}, "
                                      f"{logits.dtype} on {logits.device})")
        tokens, conf = K.sample_top_p_greedy(logits, top_p)
        return tokens, conf.unsqueeze(-1).expand(*logits.shape)

    @torch.no_grad()
    def get_draft_blocks(self, x: torch.Tensor, p: torch.Tensor,
                         mask_index: Optional[torch.Tensor] = None, start_pos: Optional[int] = None,
                         end_pos: Optional[int] = None, small_block_start: Optional[int] = None,
                         small_block_end: Optional[int] = None, **kwargs) -> List[dict]:
        """Draft blocks of the calibration graph (fastdllm_v2_generation.py:387-474) on the
        GPU (sf_draft_blocks): confidences and the needed top-k tokens of the small block's
        positions in one pass over their logits, every node's draft in one launch, one
        host sync (the reference runs a vocabulary topk per pair and syncs per node).
        Same arguments and result: dicts with 'state', 'start_pos', 'end_pos', 'node'."""
        if getattr(self, "calibration_graph", None) is None or mask_index is None:
            return []
        if not (x.is_cuda and p.is_cuda) or p.dtype not in (torch.bfloat16, torch.float32):
            raise NotImplementedError("GPU draft construction takes CUDA bf16 / fp32 logits "
                                      f"(got {p.dtype} on {p.device})")
        if small_block_start is not None and small_block_end is not None:
            lo, hi = small_block_start, small_block_end
        else:
            lo, hi = 0, x.shape[0]
        # the reference's softmax runs in the logits' dtype (:434)
        nodes, drafts, valid = self._draft_states(x, p[lo:hi], mask_index[lo:hi], lo, conf_fp32=False)
        return [{"state": drafts[k], "start_pos": start_pos, "end_pos": end_pos, "node": n}
                for k, n in enumerate(nodes) if valid[k]]


class SpecFoldB200NLDGeneration(FoldedVerifyB200):
    """Nemotron-Labs-Diffusion (Ministral3 / Llama backbone): no QKV bias, unshifted
    logits, llama-4 query scale applied in the QKV epilogue instead of falling back
    (replaces SpecFoldTritonNLDGeneration, nld_folded.py:244-394)."""

    family = "nld"

    @torch.no_grad()
    def get_draft_blocks(self, x_block: torch.Tensor, logits_block: torch.Tensor,
                         mask_index: torch.Tensor) -> List[dict]:
        """Draft blocks of the calibration graph over the whole block
        (nld_generation.py:108-151) on the GPU (sf_draft_blocks; fp32 confidences as the
        reference's softmax of logits.float()).  Dicts with 'state' and 'node'."""
        if not (x_block.is_cuda and logits_block.is_cuda) or \
                logits_block.dtype not in (torch.bfloat16, torch.float32):
            raise NotImplementedError("GPU draft construction takes CUDA bf16 / fp32 logits "
                                      f"(got {logits_block.dtype} on {logits_block.device})")
        nodes, drafts, valid = self._draft_states(x_block, logits_block, mask_index, 0, conf_fp32=True)
        return [{"state": drafts[k], "node": n} for k, n in enumerate(nodes) if valid[k]]

    def _q_scale(self, cfg, P, N, device, force=False):
        """llama-4 query scale of block positions [P, P + N) (nld_folded.py:37-53); None
        when it is identically 1, unless ``force`` (a table over a cache's capacity,
        copied from per call, must exist whenever the model has the parameters)."""
        rp = getattr(cfg, "rope_parameters", None) or {}
        beta = rp.get("llama_4_scaling_beta")
        omax = rp.get("original_max_position_embeddings")
        if beta is None or omax is None:
            return None
        pos = torch.arange(P, P + N, device=device, dtype=torch.float32)
        scale = 1.0 + beta * torch.log(1.0 + torch.floor(pos / omax))
        if not force and bool((scale == 1.0).all()):
            return None
        return scale.contiguous()
