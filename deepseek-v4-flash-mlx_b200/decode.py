"""Device-resident sparse-MLA decode state and the decode attention step.

The reference keeps the decode state on the host and rebuilds the attended rows every token:
a 128-row window ring `winr` and a growing `kvbuf` of [window rows | visible compressed rows]
uploaded per step (oracle/v4_fast.py:93-118, oracle/step12_glue.py:142-173), which its own notes
flag as the cost that grows with context (oracle/v4_serve_fast.py:116). Here the state lives in
HBM and is addressed by index:

  kv_pool     bf16 [batch*window + n_pages*page, 512]: first each sequence's window ring
              (row win_base[b] + p % window), then pages of compressed rows
  block_table int32 [batch, pages_per_seq]: compressed entry j of sequence b lives at pool row
              comp_base + block_table[b, j // page] * page + j % page
  k_idx       fp32 [batch, max_comp, 128]: indexer keys of the compressed entries
  ring_kv / ring_score fp32 [batch, 2*ratio, 1024]: the compressor's decode ring

`decode_attention` is the measured decode path: on one stream, chained with programmatic dependent
launch, the indexer scores, the top-k selection straight into the attention index list (mapped
through the block table), sparse attention — whose window tiles, computed from the positions, run
while the selection finishes — with the inverse RoPE fused into its epilogue, and the split-K merge;
q's per-head norm + RoPE is fused into the attention kernel for decode-sized batches (below 16
sequences), else it runs on a side stream beside the indexer.
"""
import ctypes
import math

import torch

from . import _lib as L
from .indexer import build_key_image, indexer_topk_into, key_image_buffers
from .norm_rope import norm_rope, rope_freqs
from .sparse_attn import sparse_attn_decode, sparse_attn_into, sparse_attn_rope

# below this batch the decode step fuses q's norm + RoPE into the attention kernel (the head-group
# kernel's prologue); from it on the norm runs on a side stream beside the indexer
FUSED_Q_MAX_BATCH = 16


class SparseMLACache:
    def __init__(self, batch, max_comp, window=128, head_dim=512, idx_dim=128, ratio=4, page=64,
                 device="cuda", page_order=None):
        self.batch, self.window, self.head_dim, self.ratio, self.page = batch, window, head_dim, ratio, page
        self.max_comp = max_comp
        self.pages_per_seq = math.ceil(max_comp / page)
        n_pages = batch * self.pages_per_seq
        self.comp_base = batch * window
        self.kv_pool = torch.zeros((self.comp_base + n_pages * page, head_dim), dtype=torch.bfloat16,
                                   device=device)
        self.win_base = (torch.arange(batch, dtype=torch.int64) * window).to(device)
        if page_order is None:
            page_order = torch.arange(n_pages, dtype=torch.int32)
        self.block_table = page_order.to(torch.int32).reshape(batch, self.pages_per_seq).to(device)
        self.image_stale = False
        # max_comp == 0: a window-only layer (ratio 0, and the ratio-128 layers, which the reference
        # runs with neither a compressor ring nor compressed rows, oracle/v4_fast.py:42-43, 114)
        self.compressed = max_comp > 0
        if not self.compressed:
            self.k_idx = self.key_image = None
            self.ring_kv = self.ring_score = self.ring_k_idx = self.ring_s_idx = None
            return
        self.k_idx = torch.zeros((batch, max_comp, idx_dim), dtype=torch.float32, device=device)
        # the indexer keys' split form for the tensor-core filter, kept current with k_idx
        self.key_image = key_image_buffers(batch, max_comp, device)
        self.ring_kv = torch.zeros((batch, 2 * ratio, 2 * head_dim), dtype=torch.float32, device=device)
        self.ring_score = torch.full((batch, 2 * ratio, 2 * head_dim), float("-inf"), dtype=torch.float32,
                                     device=device)
        self.ring_k_idx = torch.zeros((batch, 2 * ratio, 2 * idx_dim), dtype=torch.float32, device=device)
        self.ring_s_idx = torch.full((batch, 2 * ratio, 2 * idx_dim), float("-inf"), dtype=torch.float32,
                                     device=device)

    # ---- checkpoint / resume (the reference copies its per-layer state with clone_states,
    # oracle/v4_fast.py:150-159, and copy.deepcopy, oracle/decode_engine.py:167) ----
    _STATE = ("kv_pool", "win_base", "block_table", "k_idx", "key_image", "ring_kv", "ring_score", "ring_k_idx",
              "ring_s_idx")

    def state_dict(self):
        """The whole decode state as tensors (on the cache's device), for torch.save; the key image
        is saved as its three buffers."""
        st = {}
        for name in self._STATE:
            v = getattr(self, name)
            if name == "key_image" and v is not None:
                for i, t in enumerate(v):
                    st[f"key_image.{i}"] = t
            elif v is not None:
                st[name] = v
        st["meta"] = torch.tensor([self.batch, self.max_comp, self.window, self.head_dim, self.ratio, self.page,
                                   int(self.image_stale)], dtype=torch.int64)
        return st

    def load_state_dict(self, st):
        """Restore a state_dict into this cache (same shapes; copied into the existing buffers, so
        CUDA graphs captured on this cache stay valid)."""
        meta = st["meta"].tolist()
        if meta[:6] != [self.batch, self.max_comp, self.window, self.head_dim, self.ratio, self.page]:
            raise ValueError(f"SparseMLACache.load_state_dict: saved layout {meta[:6]} differs from this cache's")
        for name in self._STATE:
            v = getattr(self, name)
            if name == "key_image" and v is not None:
                for i, t in enumerate(v):
                    t.copy_(st[f"key_image.{i}"])
            elif v is not None:
                v.copy_(st[name])
        self.image_stale = bool(meta[6])

    def clone(self):
        """An independent copy of the decode state (new buffers on the same device)."""
        c = object.__new__(SparseMLACache)
        c.__dict__.update(self.__dict__)
        for name in self._STATE:
            v = getattr(self, name)
            if name == "key_image" and v is not None:
                c.key_image = tuple(t.clone() for t in v)
            elif v is not None:
                setattr(c, name, v.clone())
        return c

    # ---- address helpers (host side) ----
    def comp_rows(self, b, j):
        """Pool rows of compressed entries j (tensor) of sequence b."""
        bt = self.block_table[b].long()
        return self.comp_base + bt[j // self.page] * self.page + j % self.page

    def window_rows(self, b, positions):
        return self.win_base[b] + positions % self.window

    def fill_compressed(self, b, rows_bf16, keys_f32):
        """Place n compressed rows (and their indexer keys) of sequence b (prefill hand-off)."""
        n = rows_bf16.shape[0]
        j = torch.arange(n, device=rows_bf16.device)
        self.kv_pool[self.comp_rows(b, j)] = rows_bf16.to(torch.bfloat16)
        self.k_idx[b, :n] = keys_f32
        self.image_stale = True

    def refresh_key_image(self):
        """Rebuild the key image from k_idx (after host-side fills; decode steps keep it current)."""
        build_key_image(self.k_idx, self.key_image)
        self.image_stale = False

    def fill_window(self, b, positions, rows_bf16):
        self.kv_pool[self.window_rows(b, positions)] = rows_bf16.to(torch.bfloat16)

    def load_prefill(self, b, window_rows, comp_rows=None, keys=None, ring=None, key_ring=None):
        """Seed sequence b's decode state from a prefill of its first s tokens (positions 0..s-1),
        the state the reference's prefill leaves for its decode steps (oracle/decode_engine.py:86-95):
        window_rows [s, head_dim] are the tokens' kv rows (the last min(s, window) of them go to
        their ring slots p % window); comp_rows [n, head_dim] and keys [n, idx_dim] are the
        compressed entries 0..n-1 and their indexer keys; ring / key_ring = (ring_kv, ring_score)
        [1 or b, 2*ratio, 2*dim] are the compressors' rings after the prefill (compressor_prefill's
        state["ring_kv"], state["ring_score"]). The next decode token is at position s."""
        s = window_rows.shape[0]
        lo = max(0, s - self.window)
        pos = torch.arange(lo, s, device=self.kv_pool.device)
        self.fill_window(b, pos, window_rows[lo:s])
        if not self.compressed:
            return
        n = comp_rows.shape[0] if comp_rows is not None else 0
        if n > self.max_comp:
            raise ValueError(f"SparseMLACache.load_prefill: {n} compressed rows exceed the cache's {self.max_comp}")
        if n:
            self.fill_compressed(b, comp_rows, keys)
        # an omitted ring starts from the compressor's initial state (kv 0, scores -inf), never from
        # what a previous sequence left in slot b
        if ring is not None:
            self.ring_kv[b].copy_(ring[0].reshape(self.ring_kv[b].shape))
            self.ring_score[b].copy_(ring[1].reshape(self.ring_score[b].shape))
        else:
            self.ring_kv[b].zero_()
            self.ring_score[b].fill_(float("-inf"))
        if key_ring is not None:
            self.ring_k_idx[b].copy_(key_ring[0].reshape(self.ring_k_idx[b].shape))
            self.ring_s_idx[b].copy_(key_ring[1].reshape(self.ring_s_idx[b].shape))
        else:
            self.ring_k_idx[b].zero_()
            self.ring_s_idx[b].fill_(float("-inf"))


def decode_rows(cache, positions):
    """Pool rows of one decode step, one launch (dsv4_decode_rows): (win_rows, comp_rows, key_rows),
    int64 [b] each — this token's window slot, the compressed row the step emits (when
    (p+1) % ratio == 0) and its indexer key row in k_idx viewed as [batch*max_comp, 128]."""
    L.require_cuda(positions)
    b = positions.shape[0]
    pos = positions.to(torch.int32).contiguous()
    out = torch.empty((3, b), dtype=torch.int64, device=positions.device)
    p = L.DecodeRowsParams()
    p.positions, p.win_base, p.block_table = L.ptr(pos), L.ptr(cache.win_base), L.ptr(cache.block_table)
    p.win_rows, p.comp_rows, p.key_rows = L.ptr(out[0]), L.ptr(out[1]), L.ptr(out[2])
    p.comp_base, p.b, p.window, p.ratio, p.page = cache.comp_base, b, cache.window, cache.ratio, cache.page
    p.bt_stride, p.max_comp = cache.block_table.shape[1], cache.max_comp
    L.check(L.lib().dsv4_decode_rows(ctypes.byref(p), L.stream_of(positions)))
    return out[0], out[1], out[2]


def attention_index_buffer(batch, window, top_k, device):
    """The explicit part of a decode token's attention list: its top_k compressed pool rows (the
    window rows are computed inside the attention kernel)."""
    return torch.empty((batch, top_k), dtype=torch.int32, device=device)


@torch.library.custom_op("dsv4::decode_attention", mutates_args=("idx_buf",), device_types="cuda")
def _decode_attention_op(kv_pool: torch.Tensor, k_idx: torch.Tensor, block_table: torch.Tensor,
                         win_base: torch.Tensor, key_image: torch.Tensor | None, key_inv: torch.Tensor | None,
                         key_norm_max: torch.Tensor | None, q: torch.Tensor, q_idx: torch.Tensor, w_idx: torch.Tensor,
                         sink: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor, idx_buf: torch.Tensor,
                         top_k: int, scale: float, window: int, ratio: int, page: int, comp_base: int,
                         out_dtype: torch.dtype) -> torch.Tensor:
    b = q.shape[0]
    image = (key_image, key_inv, key_norm_max) if key_image is not None else None
    if b < FUSED_Q_MAX_BATCH:
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
        return _fused_decode_into(out, kv_pool, k_idx, block_table, win_base, image, q, q_idx, w_idx, sink, positions,
                                  freqs, idx_buf, top_k, scale, window, ratio, page, comp_base)
    return _split_decode(kv_pool, k_idx, block_table, win_base, image, q, q_idx, w_idx, sink, positions, freqs,
                         idx_buf, top_k, scale, window, ratio, page, comp_base, out_dtype)


def _split_decode(kv_pool, k_idx, block_table, win_base, image, q, q_idx, w_idx, sink, positions, freqs, idx_buf,
                  top_k, scale, window, ratio, page, comp_base, out_dtype, fetch_q=None, out=None):
    """Larger batches: q's norm + RoPE on a side stream beside the indexer, then the attention
    (split over the list, merged by the combine kernel). `fetch_q` (optional) launches work on the
    side stream before the norm (the host step's copy of q, which only the attention reads). `out`
    (optional, q's shape) receives the result, device memory or a pinned host block."""
    b = q.shape[0]
    main = torch.cuda.current_stream(q.device)
    side = _side_stream(q.device)
    side.wait_stream(main)
    with torch.cuda.stream(side):          # q's norm + rope runs beside the indexer
        if fetch_q is not None:
            fetch_q()
        qr = norm_rope(q, positions, freqs, weight=None)
    indexer_topk_into(idx_buf.view(b, 1, -1), q_idx.reshape(b, 1, *q_idx.shape[-2:]), w_idx.reshape(b, 1, -1),
                      k_idx, top_k, positions.view(b, 1), ratio, out_col=0, out_offset=comp_base,
                      block_table=block_table, page=page, key_image=image)
    main.wait_stream(side)
    qr.record_stream(main)
    if out is not None:
        return sparse_attn_into(out, qr, kv_pool, sink, idx_buf, float(scale), freqs, positions, 64, 0, False, 1e-6,
                                win_base, int(window))
    return sparse_attn_rope(qr, kv_pool, sink, idx_buf, scale, positions, freqs, 64, out_dtype,
                            win_base=win_base, window=window)


def _fused_decode_into(out, kv_pool, k_idx, block_table, win_base, image, q, q_idx, w_idx, sink, positions, freqs,
                       idx_buf, top_k, scale, window, ratio, page, comp_base, before_attention=None):
    """Decode-sized batches: one stream, three kernels chained by programmatic dependent launch
    (scores, selection, attention); q's norm + RoPE is fused into the attention kernel, which
    stores o into `out` (device memory, or a pinned host block). `before_attention` (optional)
    launches work between the selection and the attention (the host step's copy of q)."""
    b = q.shape[0]
    indexer_topk_into(idx_buf.view(b, 1, -1), q_idx.reshape(b, 1, *q_idx.shape[-2:]), w_idx.reshape(b, 1, -1),
                      k_idx, top_k, positions.view(b, 1), ratio, out_col=0, out_offset=comp_base,
                      block_table=block_table, page=page, key_image=image)
    if before_attention is not None:
        before_attention()
    # the score kernel waits for all earlier work before the selection and the attention launch,
    # so the attention may stage q and its window tiles before its own wait (pre_wait)
    return sparse_attn_into(out, q, kv_pool, sink, idx_buf, float(scale), freqs, positions, 64, 0, True, 1e-6,
                            win_base, int(window), False, 0, True)


@_decode_attention_op.register_fake
def _(kv_pool, k_idx, block_table, win_base, key_image, key_inv, key_norm_max, q, q_idx, w_idx, sink, positions, freqs,
      idx_buf, top_k, scale, window, ratio, page, comp_base, out_dtype):
    return q.new_empty(q.shape, dtype=out_dtype)


def decode_attention(cache, q, q_idx, w_idx, sink, positions, top_k=512, scale=None, freqs=None, idx_buf=None,
                     out_dtype=torch.bfloat16):
    """One decode token per sequence, through the custom op `dsv4::decode_attention`.

    q [b, 64, 512] raw (before the per-head norm), q_idx [b, 64, 128] fp32, w_idx [b, 64] fp32,
    sink [64] fp32, positions int32 [b] (position p of the new token). Returns o [b, 64, 512] after
    the inverse RoPE (the input of the output projection, oracle/v4_fast.py:118-119)."""
    L.require_cuda(q, q_idx, w_idx, sink, positions)
    b = q.shape[0]
    if scale is None:
        scale = cache.head_dim ** -0.5
    if freqs is None:
        freqs = rope_freqs(64, q.device)
    positions = positions.to(torch.int32).contiguous()
    idx = idx_buf if idx_buf is not None else attention_index_buffer(b, cache.window, top_k, q.device)
    if cache.image_stale:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("decode_attention: the cache's key image is stale inside a stream capture (the full "
                               "rebuild would replay every step); call cache.refresh_key_image() before capturing")
        cache.refresh_key_image()
    img, inv, nmax = cache.key_image if cache.key_image is not None else (None, None, None)
    return _decode_attention_op(cache.kv_pool, cache.k_idx, cache.block_table, cache.win_base, img, inv, nmax, q,
                                q_idx, w_idx, sink, positions, freqs, idx, int(top_k), float(scale),
                                int(cache.window), int(cache.ratio), int(cache.page), int(cache.comp_base), out_dtype)


def window_attention(cache, q, sink, positions, scale=None, freqs=None, idx_buf=None, out_dtype=torch.bfloat16):
    """Decode attention of a window-only layer: one token per sequence over its window ring alone
    (the ratio-0 and ratio-128 layers, oracle/v4_fast.py:110-119 with nvis = 0; the list is the
    window rows in ring order, ref_torch/sparse_attn.py:11-13). q [b, 64, 512] raw (before the
    per-head norm), sink [64], positions int32 [b] -> o [b, 64, 512] after the inverse RoPE.

    The window rows are an explicit list (dsv4_decode_window_indices), so the attention waits for
    the kernels before it (this token's row is written just before) before it reads any row."""
    L.require_cuda(q, sink, positions)
    b = q.shape[0]
    if scale is None:
        scale = cache.head_dim ** -0.5
    if freqs is None:
        freqs = rope_freqs(64, q.device)
    positions = positions.to(torch.int32).contiguous()
    idx = idx_buf if idx_buf is not None else torch.empty((b, cache.window), dtype=torch.int32, device=q.device)
    L.check(L.lib().dsv4_decode_window_indices(b, cache.window, L.ptr(positions), L.ptr(cache.win_base), L.ptr(idx),
                                               idx.shape[-1], L.stream_of(q)))
    return sparse_attn_decode(q, cache.kv_pool, sink, idx, scale, positions, freqs, 64, out_dtype=out_dtype)


_side_streams = {}


def _side_stream(device):
    key = torch.device(device).index
    st = _side_streams.get(key)
    if st is None:
        st = _side_streams[key] = torch.cuda.Stream(device)
    return st


class DecodeRunner:
    """CUDA-graph-backed decode attention for a fixed batch: the serving-loop entry point.

    The first call captures `decode_attention` on static device buffers into CUDA graphs (the
    reference's per-token path is a Python loop of library calls, oracle/v4_fast.py:82-122; here one
    graph launch replays the kernels). `step_device` replays with inputs already on the device.
    `step_host` runs a second graph that also holds the step's copies: this token's inputs from one
    pinned host block to the device (q, q_idx, w_idx and positions sit at fixed offsets of both
    blocks), the kernels, and the output back to pinned host memory, so a step is one launch. Below
    16 sequences the copies are kernels (copy kernels in, the attention kernel's own stores out); from
    16 on the inputs are copy-engine transfers, with q's beside the indexer, and the attention's merge
    kernel stores the output into the pinned tensor itself.
    Callers that write their inputs straight into `host_inputs()` skip the host-side staging copy.
    """

    def __init__(self, cache, sink, top_k=512, device="cuda", out_dtype=torch.bfloat16, stream=None,
                 q_dtype=torch.float32, keep_graph=False):
        """`q_dtype`: the dtype of q in the input block (float32, or bfloat16 to halve its copy: the
        kernels round the normed q to bf16 either way, but the per-head norm then reads bf16 values).
        `keep_graph`: keep the captured cudaGraph_t (for inspection of its nodes)."""
        if q_dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("DecodeRunner: q_dtype must be float32 or bfloat16")
        if not cache.compressed:
            raise ValueError("DecodeRunner runs the compressed layer's step (indexer + sparse attention); a window-only "
                             "cache (ratio 0 or 128) is stepped by DecodeBlock or window_attention")
        self.cache, self.top_k = cache, top_k
        b = cache.batch
        dev = torch.device(device)
        self.sink = sink.float().contiguous().to(dev)
        self.keep_graph = keep_graph
        shapes = [((b, 64, cache.head_dim), q_dtype), ((b, 64, 128), torch.float32), ((b, 64), torch.float32),
                  ((b,), torch.int32)]
        offs, total = [], 0
        for shape, dt in shapes:  # 256-byte aligned fields of one block
            offs.append(total)
            total += -(-math.prod(shape) * torch.empty((), dtype=dt).element_size() // 256) * 256
        self._in_bytes = total
        self._q_bytes = offs[1]  # q's field, padded to 256 bytes
        self.d_in = torch.zeros(total, dtype=torch.uint8, device=dev)
        self.h_in = torch.zeros(total, dtype=torch.uint8).pin_memory()

        def views(buf):
            return [buf[o:o + math.prod(sh) * torch.empty((), dtype=dt).element_size()].view(dt).view(sh)
                    for o, (sh, dt) in zip(offs, shapes)]
        self.q, self.q_idx, self.w_idx, self.positions = views(self.d_in)
        self.h_q, self.h_qi, self.h_w, self.h_pos = views(self.h_in)
        self.idx = attention_index_buffer(b, cache.window, top_k, dev)
        self.freqs = rope_freqs(64, dev)
        self.out_dtype = out_dtype
        self.out = None
        self.graph = None
        self.graph_host = None
        self.stream = stream or torch.cuda.Stream(dev)
        self.h_out = None
        self._done = None

    def _body(self):
        return decode_attention(self.cache, self.q, self.q_idx, self.w_idx, self.sink, self.positions, self.top_k,
                                freqs=self.freqs, idx_buf=self.idx, out_dtype=self.out_dtype)

    def _body_into(self, out, before_attention=None):
        c = self.cache
        image = c.key_image if c.key_image is not None else None
        return _fused_decode_into(out, c.kv_pool, c.k_idx, c.block_table, c.win_base, image, self.q, self.q_idx,
                                  self.w_idx, self.sink, self.positions, self.freqs, self.idx, self.top_k,
                                  c.head_dim ** -0.5, c.window, c.ratio, c.page, c.comp_base, before_attention)

    def capture(self):
        with torch.cuda.stream(self.stream):
            if self.cache.image_stale:   # rebuilt here, never inside the captured step
                self.cache.refresh_key_image()
            self._body()  # warm up allocations and one-time attributes outside capture
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph(keep_graph=self.keep_graph)
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.out = self._body()
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.graph_host = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph_host, stream=self.stream):
            # decode-sized batches: the step's inputs and output cross the bus by kernel loads /
            # stores of the pinned blocks, not copy-engine transfers (tens of KB, latency-bound):
            # the inputs by copy kernels (dsv4_copy), and the attention kernel stores o into the
            # pinned output itself.
            if self.cache.batch < FUSED_Q_MAX_BATCH:
                # q (the block's first field) is read only by the attention: its copy runs beside
                # the top-k selection (dsv4_copy_beside), so only q_idx, w_idx and the positions
                # cross the bus before the scores
                nq = self._q_bytes
                L.copy_(self.d_in[nq:], self.h_in[nq:])
                out = self._body_into(self.h_out,
                                      before_attention=lambda: L.copy_beside_(self.d_in[:nq], self.h_in[:nq]))
            else:
                # megabytes per step: copy-engine transfers (memcpy nodes), which take no SM (a copy
                # kernel's blocks hold the SMs in a small-shared-memory configuration, so the
                # indexer's CTAs could not start beside it). q (4 MB at batch 64) crosses on the side
                # stream, beside the indexer, which needs only q_idx, w_idx and the positions
                nq = self._q_bytes
                self.d_in[nq:].copy_(self.h_in[nq:], non_blocking=True)
                c = self.cache
                out = _split_decode(c.kv_pool, c.k_idx, c.block_table, c.win_base, c.key_image, self.q, self.q_idx,
                                    self.w_idx, self.sink, self.positions, self.freqs, self.idx, self.top_k,
                                    c.head_dim ** -0.5, c.window, c.ratio, c.page, c.comp_base, self.out_dtype,
                                    fetch_q=lambda: self.d_in[:nq].copy_(self.h_in[:nq], non_blocking=True),
                                    out=self.h_out)
        self.out_host_graph = out

    def host_inputs(self):
        """The pinned host views (q, q_idx, w_idx, positions) that `step_host` copies from."""
        return self.h_q, self.h_qi, self.h_w, self.h_pos

    def step_device(self):
        if self.graph is None:
            self.capture()
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        torch.cuda.current_stream(self.out.device).wait_stream(self.stream)
        return self.out

    def step_host(self, q, q_idx, w_idx, positions):
        """Host tensors in, host tensor out, as one graph launch on the runner's stream (input copy,
        kernels, output copy). Inputs that are not the `host_inputs()` views are first copied into
        them (after the previous step has finished with them). The returned pinned output is valid
        after `synchronize()` and until the next step."""
        if self.graph is None:
            self.capture()
        srcs = (q, q_idx, w_idx, positions)
        mine = (self.h_q, self.h_qi, self.h_w, self.h_pos)
        if not all(a.data_ptr() == b.data_ptr() and a.shape == b.shape for a, b in zip(srcs, mine)):
            if self._done is not None:
                self._done.synchronize()
            for dst, src in zip(mine, srcs):
                dst.copy_(src)
        with torch.cuda.stream(self.stream):
            self.graph_host.replay()
            if self._done is None:
                self._done = torch.cuda.Event()
            self._done.record(self.stream)
        return self.h_out

    def h2d_bytes(self):
        return self._in_bytes

    def d2h_bytes(self):
        return self.out.numel() * self.out.element_size() if self.out is not None else 0

    def synchronize(self):
        self.stream.synchronize()

    def release(self):
        """Drop the captured graphs (their memory returns to torch's graph pool)."""
        self.stream.synchronize()
        self.graph = self.graph_host = None
        self.out = self.out_host_graph = None
