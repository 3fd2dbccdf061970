"""Drop-in for MServe's ``CPUKVCache`` (qwen-eljrte/Qwen_Transformer/kv_cache.py:10-797).

Same constructor, method names, arguments and return values; different mechanics:

* host storage per layer is one pinned, device-mapped [B, H, max_len, D] allocation per
  tensor, used as a ring: appending writes only the new rows (no torch.cat + re-pin of the
  whole cache, kv_cache.py:739-759) and keeps exactly the reference's logical contents
  ("the last max_len tokens", kv_cache.py:743-748);
* ``submit_append`` writes CUDA rows straight into that host memory with the write-back
  kernel (mskv_copy_rows) on a dedicated stream ordered after the caller's stream -- there
  is no worker thread and no intermediate .cpu() copy (kv_cache.py:705-728).  The queue
  bound is kept: at most ``queue_maxsize`` appends may be in flight, beyond that the call
  returns False (block=False) or waits up to timeout_ms (block=True), as the reference's
  queue.Queue does (kv_cache.py:682-702);
* ``get_sparse_async_uva`` gathers the selected rows with the sm_100a gather kernel into new
  tensors on the caller's current stream, without the reference's torch.cuda.synchronize()
  (kv_cache.py:531); ``get_sparse_async`` runs the same kernel into reusable per-layer device
  buffers on the cache's own copy stream and returns views of them with that stream's event,
  as the reference's index_select + H2D path does (kv_cache.py:576-629).  There is no CPU
  index_select path;
* ``get_full_kv`` concatenates CUDA tensors with the row-copy kernel (two launches into one new
  tensor per K and V), as torch.cat does in the reference (kv_cache.py:631-643);
* indices are bounds-checked: a token index >= the cached length raises RuntimeError (the
  reference reads past the host tensor when the selection includes the token being
  decoded, attention.py:1953-1967).
"""
from __future__ import annotations

import threading
import time
from typing import List, Optional, Tuple

import numpy as np
import torch

from . import ops


class _Layer:
    __slots__ = ("k", "v", "B", "H", "D", "dtype", "start", "len", "version", "pending", "start_dev", "lock")

    def __init__(self, B: int, H: int, cap: int, D: int, dtype: torch.dtype):
        self.k = ops.host_empty((B, H, cap, D), dtype)
        self.v = ops.host_empty((B, H, cap, D), dtype)
        self.B, self.H, self.D, self.dtype = B, H, D, dtype
        self.start = 0          # ring slot of logical token 0 (all sequences of the batch)
        self.len = 0            # logical tokens held
        self.version = 0
        self.pending: List[torch.cuda.Event] = []
        self.start_dev = {}     # device index -> (start, int32 [B] device tensor of it)
        self.lock = threading.Lock()


def _cat_tokens(old: torch.Tensor, new: torch.Tensor) -> torch.Tensor:
    """[B, H, T, D] ++ [B, H, n, D] along tokens on the GPU with two row-copy launches."""
    if old.dim() != 4 or new.dim() != 4 or old.shape[:2] != new.shape[:2] or old.shape[3] != new.shape[3]:
        raise RuntimeError(f"Sizes of tensors must match except in dimension 2: {tuple(old.shape)} vs "
                           f"{tuple(new.shape)}")
    if old.dtype != new.dtype or old.device != new.device:
        raise RuntimeError("get_full_kv: past and new KV must share dtype and device")
    B, H, T, D = old.shape
    n = new.shape[2]
    out = torch.empty(B, H, T + n, D, dtype=old.dtype, device=old.device)
    for src, lo, cnt in ((old, 0, T), (new, T, n)):
        if cnt == 0 or B * H * D == 0:
            continue
        if src.stride(3) != 1:
            src = src.contiguous()
        ops.copy_rows(ops.strided_rows(src, device=src.device),
                      ops.strided_rows(out[:, :, lo:lo + cnt], device=out.device),
                      batch=B, num_tokens=cnt, device=out.device)
    return out


class CPUKVCache:
    """Host-offloaded KV cache with zero-copy gather/append kernels (see module docstring)."""

    def __init__(self, num_layers: int, max_len: int, queue_maxsize: int = 256, *,
                 device: Optional[torch.device] = None):
        self.num_layers = num_layers
        self.max_len = int(max_len)
        self.queue_maxsize = int(queue_maxsize)
        self.current_seq_len = 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._layers: List[Optional[_Layer]] = [None] * num_layers
        self._d2h_stream = torch.cuda.Stream(device=self.device)
        self._gpu_k_buffer: List[Optional[torch.Tensor]] = [None] * num_layers
        self._gpu_v_buffer: List[Optional[torch.Tensor]] = [None] * num_layers
        self._gpu_buffer_free_events: List[Optional[torch.cuda.Event]] = [None] * num_layers
        self._h2d_stream = torch.cuda.Stream(device=self.device)
        self._stopped = False

    # ------------------------------------------------------------------ bookkeeping
    def get_seq_len(self) -> int:
        return self.current_seq_len

    def _retire(self, layer: _Layer) -> None:
        layer.pending = [e for e in layer.pending if not e.query()]

    def _in_flight(self) -> int:
        n = 0
        for layer in self._layers:
            if layer is not None:
                self._retire(layer)
                n += len(layer.pending)
        return n

    def _wait_layer(self, layer: _Layer) -> None:
        for e in layer.pending:
            e.synchronize()
        layer.pending = []

    def _start_tensor(self, layer: _Layer, dev: torch.device) -> torch.Tensor:
        """int32 [B] device tensor of the layer's ring start (cached with its host value, so
        no call reads the device)."""
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        cached = layer.start_dev.get(idx)
        if cached is None or cached[0] != layer.start:
            t = torch.full((layer.B,), layer.start, dtype=torch.int32, device=f"cuda:{idx}")
            layer.start_dev[idx] = (layer.start, t)
            return t
        return cached[1]

    # ------------------------------------------------------------------ append (write-back)
    def submit_append(self, layer_idx: int, key_new: torch.Tensor, value_new: torch.Tensor,
                      block: bool = False, timeout_ms: float = 0.0) -> bool:
        """Appends [B, H, n, D] rows to the layer's host cache (kv_cache.py:682-702, 718-765).

        Returns False when ``queue_maxsize`` appends are already in flight and block is False
        (or the wait timed out), True once the append is enqueued.
        """
        if self._stopped:
            raise RuntimeError("CPUKVCache has been shut down")
        if key_new.dim() != 4 or value_new.shape != key_new.shape or value_new.dtype != key_new.dtype:
            raise ValueError("key_new/value_new must be matching [B, H, n, D] tensors")
        if self._in_flight() >= self.queue_maxsize:
            if not block:
                return False
            deadline = None if timeout_ms <= 0 else time.monotonic() + timeout_ms / 1000.0
            while self._in_flight() >= self.queue_maxsize:
                if deadline is not None and time.monotonic() >= deadline:
                    return False
                time.sleep(0.0002)
        B, H, n, D = key_new.shape
        layer = self._layers[layer_idx]
        if layer is None:
            layer = _Layer(B, H, self.max_len, D, key_new.dtype)
            self._layers[layer_idx] = layer
        if (B, H, D, key_new.dtype) != (layer.B, layer.H, layer.D, layer.dtype):
            raise ValueError(f"layer {layer_idx} holds [{layer.B},{layer.H},*,{layer.D}] {layer.dtype}, "
                             f"got {tuple(key_new.shape)} {key_new.dtype}")
        cap = self.max_len
        with layer.lock:
            keep = min(n, cap)                  # only the last `cap` new rows can survive
            first_new = n - keep
            total = layer.len + keep
            drop = max(0, total - cap)          # oldest tokens pushed out (kv_cache.py:743-745)
            new_start = (layer.start + drop) % cap
            dst_tok0 = layer.len - drop         # logical slot of the first kept row, after the drop
            src_k = key_new[:, :, first_new:, :]
            src_v = value_new[:, :, first_new:, :]
            if key_new.is_cuda:
                dev = key_new.device
                cur = torch.cuda.current_stream(dev)
                stream = self._d2h_stream if dev == self.device else torch.cuda.Stream(device=dev)
                stream.wait_stream(cur)
                with torch.cuda.stream(stream):
                    start_t = torch.full((B,), new_start, dtype=torch.int32, device=dev)
                    tok0_t = torch.full((B,), dst_tok0, dtype=torch.int32, device=dev)
                    src = ops.strided_rows(src_k, src_v, device=dev)
                    dst = ops.strided_rows(layer.k, layer.v, len_scalar=cap, ring_start=start_t, ring_cap=cap,
                                           tok0=tok0_t, device=dev)
                    ops.copy_rows(src, dst, batch=B, num_tokens=keep, device=dev, stream=stream)
                    ev = torch.cuda.Event()
                    ev.record(stream)
                for t in (src_k, src_v, start_t, tok0_t):
                    t.record_stream(stream)
                layer.pending.append(ev)
            else:
                # Rows already in host memory: place them in the ring on the CPU.
                slots = (new_start + dst_tok0 + np.arange(keep)) % cap
                sl = torch.from_numpy(slots)
                layer.k[:, :, sl, :] = src_k.to(layer.dtype)
                layer.v[:, :, sl, :] = src_v.to(layer.dtype)
            layer.start, layer.len = new_start, total - drop
            layer.version += 1
            self.current_seq_len = layer.len
        return True

    def append_new(self, layer_idx: int, key_new: torch.Tensor, value_new: torch.Tensor) -> None:
        """Synchronous append (the reference's worker-thread body, kv_cache.py:718-765)."""
        self.submit_append(layer_idx, key_new, value_new, block=True)
        self._wait_layer(self._layers[layer_idx])

    # ------------------------------------------------------------------ reads
    def get_snapshot(self, layer_idx: int) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor], int, int]:
        """(k, v, seq_len, version) in logical order (kv_cache.py:784-797).

        Waits for the layer's in-flight appends.  When the ring has not wrapped the tensors
        are views of the host store (pinned); otherwise a pinned logical-order copy.
        """
        layer = self._layers[layer_idx]
        if layer is None:
            return None, None, 0, 0
        self._wait_layer(layer)
        with layer.lock:
            if layer.start + layer.len <= self.max_len:
                k = layer.k[:, :, layer.start:layer.start + layer.len, :]
                v = layer.v[:, :, layer.start:layer.start + layer.len, :]
            else:
                idx = torch.from_numpy((layer.start + np.arange(layer.len)) % self.max_len)
                k = ops.host_empty((layer.B, layer.H, layer.len, layer.D), layer.dtype)
                v = ops.host_empty((layer.B, layer.H, layer.len, layer.D), layer.dtype)
                torch.index_select(layer.k, 2, idx, out=k)
                torch.index_select(layer.v, 2, idx, out=v)
            return k, v, layer.len, layer.version

    def get_sparse_async_uva(self, layer_idx: int, device: torch.device, token_indices: torch.Tensor):
        """Gathers the selected tokens into new CUDA tensors (kv_cache.py:493-543).

        token_indices: int64 [S] on the CPU (the reference contract) or an int32/int64 CUDA
        tensor [S], [B, S] or [B, H, S].  Returns (k [B, H, S, D], v, done_event) or None if
        the layer is empty.  The gather runs on the caller's current stream.
        """
        dev = self._cuda_device(device)
        return self._gather(layer_idx, dev, token_indices, torch.cuda.current_stream(dev), reuse=False)

    @staticmethod
    def _cuda_device(device) -> torch.device:
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("device must be a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        return dev

    def _sparse_buffers(self, layer_idx: int, layer: _Layer, dev: torch.device, S: int):
        """Reusable device buffers of the layer, keyed (layer, B, H, D, dtype, device) and grown
        to the largest S asked for, as the reference keys its GPU buffers (kv_cache.py:604-620)."""
        if not hasattr(self, "_sparse_gpu_buffers"):
            self._sparse_gpu_buffers = {}
        key = (layer_idx, layer.B, layer.H, layer.D, layer.dtype, dev.index)
        buf = self._sparse_gpu_buffers.get(key)
        if buf is None or buf[0].shape[2] < S:
            kb = torch.empty(layer.B, layer.H, max(S, 1), layer.D, dtype=layer.dtype, device=dev)
            buf = (kb, torch.empty_like(kb))
            self._sparse_gpu_buffers[key] = buf
        return buf

    def _gather(self, layer_idx: int, dev: torch.device, token_indices: torch.Tensor, stream: torch.cuda.Stream,
                reuse: bool):
        layer = self._layers[layer_idx]
        if layer is None:
            return None
        cur = torch.cuda.current_stream(dev)
        if stream != cur:
            stream.wait_stream(cur)       # the indices and any earlier use of the buffers
        for e in layer.pending:           # order after in-flight write-backs of this layer
            stream.wait_event(e)
        with layer.lock, torch.cuda.stream(stream):
            T, start = layer.len, layer.start
            if token_indices.device.type == "cpu":
                idx = token_indices.to(torch.int64)
                if idx.numel():
                    lo, hi = int(idx.min()), int(idx.max())
                    if lo < 0 or hi >= T:
                        raise RuntimeError(f"token index out of range [0, {T}): min {lo}, max {hi}")
                # asynchronous H2D from page-locked memory (pinned staging for pageable input;
                # torch keeps the pinned block until the copy has run): no host wait
                idx = idx.contiguous()
                if not idx.is_pinned():
                    idx = idx.pin_memory()
                idx = idx.to(dev, non_blocking=True)
            else:
                idx = token_indices.to(dev)
                if idx.dtype not in (torch.int32, torch.int64):
                    idx = idx.to(torch.int64)
            idx = idx.contiguous()
            S = idx.shape[-1]
            if reuse:
                kb, vb = self._sparse_buffers(layer_idx, layer, dev, S)
                k_out, v_out = kb[:, :, :S], vb[:, :, :S]
            else:
                k_out = torch.empty(layer.B, layer.H, S, layer.D, dtype=layer.dtype, device=dev)
                v_out = torch.empty_like(k_out)
            start_t = self._start_tensor(layer, dev)
            start_t.record_stream(stream)   # the cached tensor may be replaced while this runs
            src = ops.strided_rows(layer.k, layer.v, len_scalar=T, ring_start=start_t, ring_cap=self.max_len,
                                   device=dev)
            ops.gather(src, idx, k_out, v_out, batch=layer.B)
            done = torch.cuda.Event()
            done.record(stream)
        idx.record_stream(stream)
        return k_out, v_out, done

    def get_sparse_async(self, layer_idx: int, device: torch.device, token_indices: torch.Tensor):
        """The selected tokens in reusable device buffers (kv_cache.py:545-629).

        Same arguments and result values as get_sparse_async_uva.  As in the reference, the rows
        land in per-layer GPU buffers that the next call for the same layer (and shape)
        overwrites, the copy runs on the cache's own stream (ordered after the caller's current
        stream), and the returned event is recorded on that stream: wait on it before reading.
        The reference's CPU index_select into pinned buffers + H2D copy is replaced by the
        device gather straight from the host store; no CPU path exists.
        """
        dev = self._cuda_device(device)
        stream = self._h2d_stream if dev == self.device else torch.cuda.Stream(device=dev)
        return self._gather(layer_idx, dev, token_indices, stream, reuse=True)

    def check_errors(self) -> None:
        """Raises if a gather met an out-of-range device index (synchronises)."""
        ops.check_status(self.device, "CPUKVCache gather")

    def get_async(self, layer_idx: int, device: torch.device):
        """Whole layer -> reusable GPU buffer (kv_cache.py:241-294).

        Runs the row-copy kernel on a dedicated stream after the buffer's free event;
        returns (k_view, v_view, done_event) or None.
        """
        layer = self._layers[layer_idx]
        if layer is None:
            return None
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        buf = self._gpu_k_buffer[layer_idx]
        if buf is None or buf.device != dev or buf.dtype != layer.dtype or buf.shape[2] < layer.len:
            self._gpu_k_buffer[layer_idx] = torch.empty(layer.B, layer.H, self.max_len, layer.D, dtype=layer.dtype,
                                                        device=dev)
            self._gpu_v_buffer[layer_idx] = torch.empty_like(self._gpu_k_buffer[layer_idx])
            self._gpu_buffer_free_events[layer_idx] = None
        kb, vb = self._gpu_k_buffer[layer_idx], self._gpu_v_buffer[layer_idx]
        stream = self._h2d_stream if dev == self.device else torch.cuda.Stream(device=dev)
        free = self._gpu_buffer_free_events[layer_idx]
        for e in layer.pending:
            stream.wait_event(e)
        if free is not None:
            stream.wait_event(free)
        with torch.cuda.stream(stream):
            with layer.lock:
                T = layer.len
                start_t = self._start_tensor(layer, dev)
                start_t.record_stream(stream)   # the cached tensor may be replaced while this runs
                src = ops.strided_rows(layer.k, layer.v, len_scalar=T, ring_start=start_t, ring_cap=self.max_len,
                                       device=dev)
                dst = ops.strided_rows(kb, vb, len_scalar=T, device=dev)
                ops.copy_rows(src, dst, batch=layer.B, num_tokens=T, device=dev, stream=stream)
            done = torch.cuda.Event()
            done.record(stream)
        return kb[:, :, :T, :], vb[:, :, :T, :], done

    def mark_layer_buffer_consumed(self, layer_idx: int, stream: torch.cuda.Stream) -> None:
        """Records that the get_async buffer of a layer may be overwritten (kv_cache.py:482-491)."""
        if self._gpu_k_buffer[layer_idx] is None:
            return
        evt = torch.cuda.Event()
        evt.record(stream)
        self._gpu_buffer_free_events[layer_idx] = evt

    @staticmethod
    def get_full_kv(past_key_value: Optional[Tuple[torch.Tensor, torch.Tensor]], key_new: torch.Tensor,
                    value_new: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """cat(past, new) along the token axis (kv_cache.py:631-643): [B, H, T, D] + [B, H, n, D]
        -> new tensors [B, H, T + n, D].

        For CUDA tensors the rows are moved by the row-copy kernel (mskv_copy_rows: the past
        rows, then the new ones behind them, on the current stream; any strides with a
        contiguous head_dim).  Host tensors are concatenated by torch, as in the reference.
        """
        if past_key_value is None:
            return key_new, value_new
        k_old, v_old = past_key_value
        if not all(t.is_cuda for t in (k_old, v_old, key_new, value_new)):
            return torch.cat([k_old, key_new], dim=2), torch.cat([v_old, value_new], dim=2)
        return _cat_tokens(k_old, key_new), _cat_tokens(v_old, value_new)

    def shutdown(self, wait: bool = False, drain: bool = True, timeout_s: Optional[float] = None) -> None:
        """Drains in-flight appends (drain=True) and refuses further appends (kv_cache.py:769-781)."""
        if drain or wait:
            deadline = None if timeout_s is None else time.monotonic() + timeout_s
            for layer in self._layers:
                if layer is None:
                    continue
                while layer.pending:
                    if deadline is not None and time.monotonic() > deadline:
                        break
                    self._retire(layer)
                    if layer.pending:
                        time.sleep(0.0002)
        self._stopped = True
