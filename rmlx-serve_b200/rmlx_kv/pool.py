"""Device paged KV pool (rmlx_kv_pool_* / rmlx_kv_* entry points).

Arguments that name device memory accept a torch tensor (its data pointer is
passed; torch only owns the memory) or a raw integer device address.  The
stream defaults to torch's current stream on the pool's device.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

from . import _lib
from ._lib import check, lib

F32, F16, BF16 = _lib.F32, _lib.F16, _lib.BF16


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream, device: int) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream(device).cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


@dataclass
class PoolLayout:
    base: int
    bytes: int
    tile_bytes: int
    block_bytes: int
    row_bytes: int
    meta_row_bytes: int


class KVPool:
    """Block-major paged KV pool on one GPU: pool[block][layer][kv][head][slot][row]."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, block_size: int, num_blocks: int,
                 dtype: int = BF16, quant_bits: int = 0, group_size: int = 64, meta_dtype: int = F32,
                 head_offset: int = 0, device: int = 0):
        cfg = _lib.PoolConfig(num_layers, num_kv_heads, head_dim, block_size, num_blocks, dtype, quant_bits,
                              group_size, meta_dtype, head_offset)
        h = _lib.vp()
        check(lib.rmlx_kv_pool_new(C.byref(cfg), device, C.byref(h)))
        self._h = h
        self.cfg = cfg
        self.device = device
        lay = _lib.PoolLayout()
        check(lib.rmlx_kv_pool_layout(h, C.byref(lay)))
        self.layout = PoolLayout(lay.base, lay.bytes, lay.tile_bytes, lay.block_bytes, lay.row_bytes,
                                 lay.meta_row_bytes)

    def close(self):
        if getattr(self, "_h", None):
            lib.rmlx_kv_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def check(self) -> int:
        """Synchronise and return (then clear) the device error word."""
        e = C.c_int32()
        check(lib.rmlx_kv_pool_check(self._h, C.byref(e)))
        return e.value

    def status_async(self, word, stream=None) -> None:
        """Queue a copy of the device error word into `word` (pinned host
        int32, a torch tensor or an address) on `stream`; nothing waits and
        the word is not cleared.  Read `word` once an event recorded after
        this call has completed."""
        check(lib.rmlx_kv_pool_status_async(self._h, _ptr(word), _stream(stream, self.device)))

    def read(self, offset: int = 0, nbytes: Optional[int] = None):
        """Copy pool bytes [offset, offset+nbytes) to a new host numpy array."""
        import numpy as np
        n = self.layout.bytes - offset if nbytes is None else nbytes
        out = np.empty(n, dtype=np.uint8)
        check(lib.rmlx_kv_pool_read(self._h, offset, n, out.ctypes.data))
        return out

    def write(self, data, offset: int = 0) -> None:
        """Copy a host buffer (numpy array) into the pool at `offset`."""
        import numpy as np
        a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        check(lib.rmlx_kv_pool_write(self._h, offset, a.size, a.ctypes.data))

    def append(self, k, v, slot_mapping, num_tokens: int, layer_begin: int = 0, num_layers: Optional[int] = None,
               layer_stride: Optional[int] = None, token_stride: Optional[int] = None,
               head_stride: Optional[int] = None, stream=None) -> None:
        """k/v rows (l, t, h) at element (l*layer_stride + t*token_stride + h*head_stride).

        Defaults describe a contiguous [layers][tokens][heads][head_dim] input.
        """
        c = self.cfg
        nl = c.num_layers - layer_begin if num_layers is None else num_layers
        hs = c.head_dim if head_stride is None else head_stride
        ts = c.num_kv_heads * c.head_dim if token_stride is None else token_stride
        ls = num_tokens * c.num_kv_heads * c.head_dim if layer_stride is None else layer_stride
        check(lib.rmlx_kv_append(self._h, layer_begin, nl, _ptr(k), _ptr(v), ls, ts, hs, _ptr(slot_mapping),
                                 num_tokens, _stream(stream, self.device)))

    def gather(self, layer: int, block_tables, block_table_stride: int, seq_lens, num_seqs: int, out_k, out_v,
               stream=None) -> None:
        check(lib.rmlx_kv_gather(self._h, layer, _ptr(block_tables), block_table_stride, _ptr(seq_lens),
                                 num_seqs, _ptr(out_k), _ptr(out_v), _stream(stream, self.device)))

    def gather_layers(self, layer_begin: int, num_layers: int, block_tables, block_table_stride: int, seq_lens,
                      num_seqs: int, out_k, out_v, out_layer_stride: int, stream=None) -> None:
        """Layers [layer_begin, layer_begin + num_layers) in one launch; layer
        layer_begin + i at element offset i * out_layer_stride of out_k/out_v."""
        check(lib.rmlx_kv_gather_layers(self._h, layer_begin, num_layers, _ptr(block_tables), block_table_stride,
                                        _ptr(seq_lens), num_seqs, _ptr(out_k), _ptr(out_v), out_layer_stride,
                                        _stream(stream, self.device)))

    def attention_workspace_size(self, q_heads_per_kv: int, num_seqs: int, max_total_tokens: int) -> int:
        n = C.c_size_t()
        check(lib.rmlx_kv_attention_workspace_size(self._h, q_heads_per_kv, num_seqs, max_total_tokens, C.byref(n)))
        return n.value

    def decode_attention(self, layer: int, q, q_heads_per_kv: int, block_tables, block_table_stride: int, seq_lens,
                         num_seqs: int, softmax_scale: float, out, workspace, workspace_bytes: int = None,
                         stream=None) -> None:
        """out = softmax(scale * q K^T) V per (sequence, query head), reading
        the pool's tiles through the block table (no gathered copy)."""
        if workspace_bytes is None:
            workspace_bytes = workspace.numel() * workspace.element_size()
        check(lib.rmlx_kv_decode_attention(self._h, layer, _ptr(q), q_heads_per_kv, _ptr(block_tables),
                                           block_table_stride, _ptr(seq_lens), num_seqs, softmax_scale, _ptr(out),
                                           _ptr(workspace), workspace_bytes, _stream(stream, self.device)))

    def gather_ring(self, layer: int, block_tables, block_table_stride: int, seq_lens, ring_offsets, num_seqs: int,
                    keep: int, max_size: int, out_k, out_v, stream=None) -> None:
        """Logical-order gather of ring sequences (rotating_cache.rs:162-197)."""
        check(lib.rmlx_kv_gather_ring(self._h, layer, _ptr(block_tables), block_table_stride, _ptr(seq_lens),
                                      _ptr(ring_offsets), num_seqs, keep, max_size, _ptr(out_k), _ptr(out_v),
                                      _stream(stream, self.device)))

    def move_rows(self, src_slots, dst_slots, n: int, stream=None) -> None:
        check(lib.rmlx_kv_move_rows(self._h, _ptr(src_slots), _ptr(dst_slots), n, _stream(stream, self.device)))

    def copy_blocks(self, src, dst, n: int, stream=None) -> None:
        check(lib.rmlx_kv_copy_blocks(self._h, _ptr(src), _ptr(dst), n, _stream(stream, self.device)))

    def pack_blocks(self, ids, n: int, staging, stream=None) -> None:
        check(lib.rmlx_kv_pack_blocks(self._h, _ptr(ids), n, _ptr(staging), _stream(stream, self.device)))

    def unpack_blocks(self, ids, n: int, staging, stream=None) -> None:
        check(lib.rmlx_kv_unpack_blocks(self._h, _ptr(ids), n, _ptr(staging), _stream(stream, self.device)))

    def migrate(self, comm, peer: int, send_ids, n_send: int, send_staging, recv_ids, n_recv: int, recv_staging,
                stream=None) -> None:
        """Send blocks to `peer` and receive blocks from it (both ranks call this)."""
        check(lib.rmlx_kv_migrate(self._h, comm.handle, peer, _ptr(send_ids), n_send, _ptr(send_staging),
                                  _ptr(recv_ids), n_recv, _ptr(recv_staging), _stream(stream, self.device)))


class NcclComm:
    """NCCL communicator for block migration (one process per GPU).

    Rank 0 makes the id with ``NcclComm.unique_id()`` and shares it with the
    other ranks (any host channel); every rank then constructs the comm.
    """

    def __init__(self, nranks: int, uid: bytes, rank: int, device: int, timeout_ms: int = 60000):
        if len(uid) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        h = _lib.vp()
        check(lib.rmlx_nccl_comm_new(nranks, buf, rank, device, timeout_ms, C.byref(h)))
        self._h, self.rank, self.nranks, self.device = h, rank, nranks, device

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * 128)()
        check(lib.rmlx_nccl_unique_id(buf))
        return bytes(buf)

    @property
    def handle(self):
        return self._h

    def wait(self, stream=None, timeout_ms: int = 0) -> None:
        check(lib.rmlx_nccl_wait(self._h, _stream(stream, self.device), timeout_ms))

    def close(self):
        if getattr(self, "_h", None):
            lib.rmlx_nccl_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def hash_block_chains(tokens, cu_tokens, root_hashes, num_requests: int, block_size: int, cu_blocks, out,
                      stream=None, device: int = 0) -> None:
    """Chain hashes of every block of every request (device arrays)."""
    check(lib.rmlx_hash_block_chains(_ptr(tokens), _ptr(cu_tokens), _ptr(root_hashes), num_requests, block_size,
                                     _ptr(cu_blocks), _ptr(out), _stream(stream, device)))
