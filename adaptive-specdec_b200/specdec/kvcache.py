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
"""
import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from specdec import _lib as L

__all__ = ["RaggedCache"]


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
        super().__init__(layers=[_RaggedLayer(self) for _ in range(n_layers)])

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
