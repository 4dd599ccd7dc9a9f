"""A KV cache whose rows roll back independently, in O(1), on the device.

Drop-in for the reference's specdec/kvcache.py (RaggedCache, kvcache.py:
98-202): same constructor, same geometry and mutation methods, and the
transformers ``Cache`` interface.  What changes is where the bookkeeping runs:

* ``lengths`` is device-resident and authoritative.  advance / rollback /
  commit are one tiny kernel each (sd_kv_lengths_update / sd_kv_commit): no
  data movement and no host synchronisation, also when the counts are a CUDA
  tensor (the reference copies them to the host, kvcache.py:183-185).
* a host mirror of the lengths is kept whenever the host knows them (int or
  list arguments), so ``max_len`` / ``kv_len_for`` stay sync-free on those
  paths; after a device-side rollback it is refreshed lazily, once.
* ``layers[i].update`` appends the new K/V rows at each row's own offset with
  one kernel (sd_kv_append), replacing the two scatters of kvcache.py:61-74.

Two attention modes:

* ``attn_impl="specdec_b200"`` (what the engine uses): ``update`` returns the
  full [B, Hkv, C, D] buffers and the registered attention function reads only
  each row's live keys with the verify-attention kernel (sd_verify_attn);
* the default mode returns [:, :, :max_len+q] views exactly like the reference,
  for use with stock attention implementations and ``attn_mask``.

Invariant (the reference's, kvcache.py:17-21): after a rollback the cache is
indistinguishable from one that only ever processed the accepted prefix.

``PagedRaggedCache`` keeps the same interface over pages of PAGE tokens
drawn from one pool per layer, so that memory follows each row's own length
rather than the widest row's (the reference pads every row to the capacity,
kvcache.py:98-116).
"""
import numpy as np
import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from specdec import _lib as L

__all__ = ["RaggedCache", "PagedRaggedCache", "PAGE"]

PAGE = 128            # tokens per page (SD_KV_PAGE): one K/V tile of the verify attention


class _RaggedLayer(CacheLayerMixin):
    """One layer's preallocated [B, Hkv, C, D] K and V buffers."""

    is_sliding = False
    is_compileable = False

    def __init__(self, parent):
        super().__init__()
        self.parent = parent
        self.keys = None
        self.values = None
        self.is_initialized = False

    def lazy_initialization(self, key_states, value_states=None):
        p = self.parent
        b, h, _, d = key_states.shape
        self.dtype, self.device = key_states.dtype, key_states.device
        self.keys = torch.zeros(b, h, p.capacity, d, dtype=self.dtype, device=self.device)
        self.values = torch.zeros(b, h, p.capacity, d, dtype=self.dtype, device=self.device)
        self.keys._sd_cache = p
        self.values._sd_cache = p
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        p = self.parent
        b, h, q, d = key_states.shape
        # offsets are the lengths BEFORE this forward; the parent advances once,
        # after every layer has written (kvcache.py:63-66)
        L.require_cuda(key_states, value_states, p.lengths)
        ks, vs = key_states, value_states
        if ks.stride(-1) != 1:
            ks = ks.contiguous()
        if vs.stride() != ks.stride():
            vs = vs.contiguous()
            ks = ks.contiguous()
        code = L.dtype_code(ks.dtype)
        with torch.cuda.device(ks.device):
            L.check(L.lib().sd_kv_append(L.ptr(self.keys), L.ptr(self.values), L.ptr(ks), L.ptr(vs),
                                         ks.stride(0), ks.stride(1), ks.stride(2), L.ptr(p.lengths),
                                         b, h, p.capacity, d, q, code, L.ptr(p._err),
                                         L.stream_ptr(ks.device)), "kv_append")
        p._last_q = q
        if p.attn_impl == "specdec_b200":
            return self.keys, self.values
        kv_len = p.kv_len_for(q)
        return self.keys[:, :, :kv_len, :], self.values[:, :, :kv_len, :]

    def get_mask_sizes(self, query_length, layer_idx=None):
        return self.parent.get_mask_sizes(query_length, layer_idx)

    def get_seq_length(self):
        return self.parent.get_seq_length() if self.is_initialized else 0

    def get_max_cache_shape(self):
        return self.parent.capacity


class RaggedCache(Cache):
    """Per-row-length KV cache with O(1), device-side rollback.

    Usage per forward (as the reference):
        pos  = cache.positions(q)                  # [B, q] RoPE positions
        mask = cache.attn_mask(q, dtype, valid)    # only for stock attention
        out  = model(input_ids, position_ids=pos, attention_mask=mask,
                     past_key_values=cache, cache_position=cache.cache_position(q))
        cache.advance(q)                           # exactly once per forward
    """

    _layer_cls = _RaggedLayer

    def __init__(self, n_layers, batch_size, capacity, device, attn_impl=None):
        self.capacity = int(capacity)
        self.batch_size = int(batch_size)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise L.SpecdecError("RaggedCache keeps its lengths on the GPU (no CPU fallback)")
        self.attn_impl = attn_impl
        self.lengths = torch.zeros(self.batch_size, dtype=torch.long, device=self.device)
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._host = torch.zeros(self.batch_size, dtype=torch.long)
        self._host_valid = True
        self.valid = None           # optional [B] cap for right-padded prefill
        self._last_q = 0
        super().__init__(layers=[self._layer_cls(self) for _ in range(n_layers)])

    # ---- host mirror -----------------------------------------------------
    def _mirror(self):
        if not self._host_valid:
            self._host = self.lengths.to("cpu")
            self._host_valid = True
        return self._host

    def invalidate_host(self):
        """Forget the host mirror (the next host read syncs once).  Steps that
        are replayed from CUDA graphs change the device lengths only."""
        self._host_valid = False

    @property
    def lengths_cpu(self):
        return self._mirror()

    @property
    def max_len(self):
        return int(self._mirror().max()) if self.batch_size else 0

    @property
    def _uniform(self):
        h = self._mirror()
        return bool(int(h.min()) == int(h.max()))

    # ---- geometry ----------------------------------------------------------
    def kv_len_for(self, q):
        """Width of the key/value window the stock attention path reads."""
        return self.max_len + q

    def positions(self, q):
        """RoPE positions [B, q]: each row continues from its own length."""
        ar = torch.arange(q, device=self.device).view(1, q)
        return self.lengths.view(-1, 1) + ar

    def cache_position(self, q):
        """Shared 1-D cache_position, consistent with the widest row.

        Only mask construction reads it; the kernel path builds no mask, so
        there it is arange(q) and needs no host copy of the lengths.
        """
        if self.attn_impl == "specdec_b200":
            return torch.arange(q, device=self.device)
        m = self.max_len
        return torch.arange(m, m + q, device=self.device)

    def attn_mask(self, q, dtype, valid=None):
        """Additive mask [B, 1, q, kv_len] (0 = attend) for stock attention.

        Same rule as the reference (kvcache.py:138-162): s <= lengths[b] + j,
        and s < valid[b] when given; None when all rows are level and there is
        no padding.  The kernel attention path needs no mask.
        """
        if self.attn_impl == "specdec_b200":
            self.valid = valid
            return None
        if valid is None and self._uniform:
            return None
        kv_len = self.kv_len_for(q)
        s = torch.arange(kv_len, device=self.device).view(1, 1, kv_len)
        j = torch.arange(q, device=self.device).view(1, q, 1)
        allowed = s <= (self.lengths.view(-1, 1, 1) + j)
        if valid is not None:
            allowed = allowed & (s < valid.to(self.device).view(-1, 1, 1))
        neg = torch.finfo(dtype).min
        return torch.where(allowed, 0.0, neg).to(dtype).unsqueeze(1)

    # ---- mutation ----------------------------------------------------------
    def _update(self, delta, q, sign):
        with torch.cuda.device(self.device):
            L.check(L.lib().sd_kv_lengths_update(L.ptr(self.lengths), L.ptr(delta), int(q), sign,
                                                 self.batch_size, self.capacity, L.ptr(self._err),
                                                 L.stream_ptr(self.device)), "kv lengths")

    def advance(self, q):
        """Call once per forward, after the model has run."""
        q = int(q)
        if self._host_valid and int(self._host.max()) + q > self.capacity:
            raise RuntimeError("RaggedCache.advance beyond capacity")
        self._update(None, q, +1)
        if self._host_valid:
            self._host += q
        self.valid = None

    def set_lengths(self, lengths):
        self.valid = None
        t = torch.as_tensor(lengths, dtype=torch.long)
        if t.is_cuda:
            self.lengths.copy_(t)
            self._host_valid = False
        else:
            self._host = t.clone()
            self._host_valid = True
            self.lengths.copy_(t, non_blocking=False)

    def set_host_lengths(self, lengths):
        """Tell the cache its device lengths, as the caller read them back
        (no device work): host-side geometry and page reservations then need
        no sync of their own."""
        self._host = torch.as_tensor(lengths, dtype=torch.long).reshape(-1).clone()
        self._host_valid = True

    def rollback(self, n):
        """Drop the last n[b] tokens of row b.  O(1): no copy, no allocation.

        int / list: checked on the host (RuntimeError below zero, as the
        reference, kvcache.py:188-189).  CUDA tensor: applied on the device
        with no sync; a row that would go below zero is left unchanged and
        flagged, and the next check_errors() raises.
        """
        if torch.is_tensor(n) and n.is_cuda:
            d = n.to(torch.long).reshape(-1).contiguous()
            self._update(d, 0, -1)
            self._host_valid = False
            return
        if isinstance(n, int):
            n_cpu = torch.full((self.batch_size,), n, dtype=torch.long)
        elif torch.is_tensor(n):
            n_cpu = n.detach().to("cpu", torch.long).reshape(-1)
        else:
            n_cpu = torch.as_tensor(list(n), dtype=torch.long)
        h = self._mirror()
        if bool(((h - n_cpu) < 0).any()):
            raise RuntimeError("RaggedCache.rollback below zero")
        self._update(n_cpu.to(self.device, non_blocking=True), 0, -1)
        self._host = h - n_cpu

    def commit(self, n_acc, k):
        """Verify-round commit: lengths -= k - n_acc (device n_acc, no sync)."""
        with torch.cuda.device(self.device):
            L.check(L.lib().sd_kv_commit(L.ptr(self.lengths), L.ptr(n_acc.to(torch.long)), int(k),
                                         self.batch_size, L.ptr(self._err),
                                         L.stream_ptr(self.device)), "kv commit")
        self._host_valid = False

    def check_errors(self):
        """Raise if any device-side update was refused (syncs once)."""
        if int(self._err.item()):
            self._err.zero_()
            raise RuntimeError("RaggedCache: a length update left [0, capacity]")

    # ---- Cache interface ---------------------------------------------------
    def get_seq_length(self, layer_idx: int = 0):
        # On the kernel path transformers only feeds this to mask construction,
        # which the registered mask function skips: answer from the host mirror
        # when it is valid and never read the device lengths back (so forwards
        # stay free of host syncs and can be graph-captured).
        if self.attn_impl == "specdec_b200":
            return int(self._host.max()) if self._host_valid and self.batch_size else 0
        return self.max_len

    def get_mask_sizes(self, query_length, layer_idx=0):
        # transformers 5.x passes an int query length; older callers pass the
        # cache_position tensor (the reference's signature, kvcache.py:76-78).
        # The kernel path builds no mask, so it needs no (host) max length.
        q = query_length if isinstance(query_length, int) else int(query_length.shape[0])
        if self.attn_impl == "specdec_b200":
            return q, 0
        return self.kv_len_for(q), 0

    def reset(self):
        self.lengths.zero_()
        self._host = torch.zeros(self.batch_size, dtype=torch.long)
        self._host_valid = True
        self._err.zero_()
        for layer in self.layers:
            if layer.is_initialized:
                layer.keys.zero_()
                layer.values.zero_()


class _PagedLayer(_RaggedLayer):
    """One layer's K and V page pools [n_pages, Hkv, PAGE, D]."""

    def lazy_initialization(self, key_states, value_states=None):
        p = self.parent
        _, h, _, d = key_states.shape
        self.dtype, self.device = key_states.dtype, key_states.device
        self.keys = torch.zeros(p.n_pages, h, PAGE, d, dtype=self.dtype, device=self.device)
        self.values = torch.zeros(p.n_pages, h, PAGE, d, dtype=self.dtype, device=self.device)
        self.keys._sd_cache = p
        self.values._sd_cache = p
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        p = self.parent
        b, h, q, d = key_states.shape
        L.require_cuda(key_states, value_states, p.lengths)
        ks, vs = key_states, value_states
        if ks.stride(-1) != 1:
            ks = ks.contiguous()
        if vs.stride() != ks.stride():
            vs, ks = vs.contiguous(), ks.contiguous()
        with torch.cuda.device(ks.device):
            L.check(L.lib().sd_kv_append_paged(
                L.ptr(self.keys), L.ptr(self.values), L.ptr(ks), L.ptr(vs), ks.stride(0),
                ks.stride(1), ks.stride(2), L.ptr(p.block_table), p.pages_per_row, p.n_pages,
                L.ptr(p.lengths), b, h, d, q, L.dtype_code(ks.dtype), L.ptr(p._err),
                L.stream_ptr(ks.device)), "kv_append_paged")
        p._last_q = q
        return self.keys, self.values


class PageTable:
    """Host-side page bookkeeping of a PagedRaggedCache (no device state).

    ``bt`` [B, pages_per_row] int32 holds row b's pages in slot order (-1 =
    none); pages [0, n_pages - 1) are handed out from a free stack, page
    n_pages - 1 is the sink that a right-padded prefill writes its padding
    to.  Every method returns True when ``bt`` changed.
    """

    def __init__(self, batch_size, pages_per_row, n_pages):
        if n_pages < 2:
            raise L.SpecdecError("a page pool needs at least two pages (one is the sink)")
        self.B, self.W, self.n_pages = int(batch_size), int(pages_per_row), int(n_pages)
        self.sink = self.n_pages - 1
        self.bt = np.full((self.B, self.W), -1, dtype=np.int32)
        self.owned = np.zeros(self.B, dtype=np.int64)              # real pages per row
        self.free = list(range(self.sink - 1, -1, -1))             # stack, page 0 on top

    def grow(self, need):
        """Give row b pages until it owns need[b] (slots [0, need[b] * PAGE))."""
        need = np.asarray(need, dtype=np.int64)
        if int(need.max(initial=0)) > self.W:
            raise RuntimeError("KV pages beyond the row capacity")
        short = np.maximum(need - self.owned, 0)
        total = int(short.sum())
        if total == 0:
            return False
        if total > len(self.free):
            raise L.SpecdecError(f"KV page pool exhausted: {total} pages wanted, "
                                 f"{len(self.free)} free of {self.n_pages - 1}")
        for b in np.nonzero(short)[0]:
            o = int(self.owned[b])
            for j in range(o, o + int(short[b])):
                self.bt[b, j] = self.free.pop()
            self.owned[b] = o + int(short[b])
        return True

    def reserve(self, lengths, q):
        """Pages for slots [0, lengths[b] + q) of every row."""
        lens = np.asarray(lengths, dtype=np.int64)
        return self.grow(-(-(lens + int(q)) // PAGE))

    def reserve_prefill(self, lengths, P, plen):
        """Real pages for [0, lengths[b] + plen[b]), the sink for the rest of
        [0, lengths[b] + P)."""
        lens = np.asarray(lengths, dtype=np.int64)
        pl = np.asarray(plen, dtype=np.int64)
        top = -(-(lens + int(P)) // PAGE)
        if int(top.max(initial=0)) > self.W:
            raise RuntimeError("KV pages beyond the row capacity")
        self.grow(-(-(lens + np.minimum(pl, int(P))) // PAGE))
        for b in range(self.B):
            o = int(self.owned[b])
            if top[b] > o:
                self.bt[b, o:top[b]] = self.sink
        return True

    def unsink(self):
        hit = self.bt == self.sink
        if not hit.any():
            return False
        self.bt[hit] = -1
        return True

    def release(self, rows):
        """Return the pages of the given rows to the free stack."""
        changed = False
        for b in (int(r) for r in rows):
            o = int(self.owned[b])
            self.free.extend(int(x) for x in self.bt[b, :o][::-1])
            changed = changed or o > 0 or bool((self.bt[b] >= 0).any())
            self.bt[b, :] = -1
            self.owned[b] = 0
        return changed

    def reset(self):
        self.bt[:] = -1
        self.owned[:] = 0
        self.free = list(range(self.sink - 1, -1, -1))
        return True

    def check(self):
        """Invariant: every handed-out page belongs to exactly one row slot."""
        used = self.bt[(self.bt >= 0) & (self.bt != self.sink)]
        assert len(set(used.tolist())) == used.size, "a page is owned twice"
        assert used.size + len(self.free) == self.n_pages - 1, "pages lost"
        for b in range(self.B):
            o = int(self.owned[b])
            assert (self.bt[b, :o] >= 0).all() and (self.bt[b, :o] != self.sink).all()


class PagedRaggedCache(RaggedCache):
    """RaggedCache whose rows own pages of PAGE tokens from a shared pool.

    Row b's slot s lives in page ``block_table[b, s // PAGE]`` of every
    layer's pool.  Pages are handed out on the host, before the forwards that
    need them: ``reserve(q)`` gives each row the pages for its next q tokens
    (one small host-to-device copy of the table when anything changed; no
    host sync while the host mirror of the lengths is valid), and
    ``reserve_prefill(P, plen)`` does the same for a right-padded prefill,
    pointing the padding past each row's own prompt at a shared sink page
    that nothing reads.  Pages stay with their row after a rollback (the row
    grows back into them); ``release(rows)`` and ``reset()`` return them.
    A slot written without a page sets the device error flag (bit 1).

    Only the kernel attention path (attn_impl "specdec_b200") reads paged
    layers.
    """

    _layer_cls = _PagedLayer

    def __init__(self, n_layers, batch_size, capacity, device, attn_impl="specdec_b200",
                 n_pages=None):
        if attn_impl != "specdec_b200":
            raise L.SpecdecError("PagedRaggedCache is read by the specdec_b200 attention only")
        self.pages_per_row = -(-int(capacity) // PAGE)
        super().__init__(n_layers, batch_size, self.pages_per_row * PAGE, device, attn_impl)
        self.n_pages = int(n_pages) if n_pages is not None else \
            self.batch_size * self.pages_per_row + 1
        self.pages = PageTable(self.batch_size, self.pages_per_row, self.n_pages)
        self.block_table = torch.full((self.batch_size, self.pages_per_row), -1,
                                      dtype=torch.int32, device=self.device)

    # ---- pages -------------------------------------------------------------
    @property
    def free_pages(self):
        return len(self.pages.free)

    def _push(self, changed=True):
        if changed:
            self.block_table.copy_(torch.from_numpy(self.pages.bt))

    def reserve(self, q):
        """Pages for the next q tokens of every row (call before the forward)."""
        self._push(self.pages.reserve(self._mirror().numpy(), q))

    def reserve_prefill(self, P, plen):
        """Pages for a right-padded prefill of P tokens with prompt lengths
        plen (real pages for each row's prompt, the sink for its padding)."""
        pl = torch.as_tensor(plen).to("cpu", torch.long).reshape(-1).numpy()
        self._push(self.pages.reserve_prefill(self._mirror().numpy(), P, pl))

    def release(self, rows):
        """Return the pages of the given rows to the pool (their lengths go to 0)."""
        rows = [int(r) for r in rows]
        h = self._mirror().clone()
        h[rows] = 0
        self.pages.release(rows)
        self.set_lengths(h)
        self._push()

    def set_lengths(self, lengths):
        super().set_lengths(lengths)
        self._push(self.pages.unsink())

    def reset(self):
        super().reset()
        self._push(self.pages.reset())

    def check_errors(self):
        e = int(self._err.item())
        if e:
            self._err.zero_()
            if e & 2:
                raise RuntimeError("PagedRaggedCache: a slot was written without a page "
                                   "(reserve() before the forward)")
            raise RuntimeError("RaggedCache: a length update left [0, capacity]")

    @property
    def kv_bytes(self):
        """Bytes held by the K and V pools of the initialised layers."""
        return sum(2 * l.keys.numel() * l.keys.element_size() for l in self.layers
                   if l.is_initialized)
