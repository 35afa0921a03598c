"""Oracle for the paged KV cache (test infrastructure).

BlockManagerModel restates include/BlockManager.h:29-95:
  * one pool of num_blocks * tokens_per_block * token_byte_size bytes (36-44)
  * block i starts at pool + i * tokens_per_block * token_byte_size (46-49, 79-81)
  * the free list starts as [0, 1, ..., N-1]; allocate pops from the back, so
    the first id handed out is N-1 (63-71); free pushes to the back (LIFO
    reuse, 73-82); allocating from an empty pool and freeing an id outside
    [0, N) raise (65-67, 75-77).

block_table_for_capture restates the per-capture allocation of
src/GraphWrapper.cpp:139-145: ceil(seq_len / tokens_per_block) blocks.

scatter_kv places each token's K and V head vectors.  The reference defines a
token's byte size (4096 = 8 KV heads x 128 x {K,V} x 2 bytes, see
src/GraphWrapper.cpp:41) but no layout inside a token; this build declares
[block][token_in_block][K|V][kv_head][head_dim], bf16, and the CUDA kernels
write exactly that.
"""
import numpy as np


class BlockManagerModel:
    def __init__(self, num_blocks, tokens_per_block, token_byte_size):
        self.num_blocks = num_blocks
        self.tokens_per_block = tokens_per_block
        self.token_byte_size = token_byte_size
        self.free = list(range(num_blocks))

    @property
    def pool_bytes(self):
        return self.num_blocks * self.tokens_per_block * self.token_byte_size

    def block_offset(self, block_id):
        return block_id * self.tokens_per_block * self.token_byte_size

    def allocate_block(self):
        if not self.free:
            raise RuntimeError("Out of KV Cache blocks! Massive pool exhausted.")
        return self.free.pop()

    def free_block(self, block_id):
        if block_id < 0 or block_id >= self.num_blocks:
            raise RuntimeError(
                f"BlockManager::free_block: block ID {block_id} out of range [0, {self.num_blocks})")
        self.free.append(block_id)


def block_table_for_capture(bm, seq_len, table=None):
    """src/GraphWrapper.cpp:139-145."""
    table = [] if table is None else table
    need = (seq_len + bm.tokens_per_block - 1) // bm.tokens_per_block
    for _ in range(len(table), need):
        table.append(bm.allocate_block())
    return table


def slot_of(block_table, seq, pos, tokens_per_block):
    """Physical token slot: block_table[seq][pos // B] * B + pos % B."""
    return int(block_table[seq][pos // tokens_per_block]) * tokens_per_block + pos % tokens_per_block


def scatter_kv(pool, k_bits, v_bits, block_table, token_seq, positions):
    """Write K/V rows into a pool viewed as uint16 [num_blocks, B, 2, Hkv, hd].

    k_bits, v_bits  uint16 [T, Hkv, hd] (bf16 bit patterns)
    block_table     int [num_seqs, max_blocks]
    token_seq, positions  int [T]
    Returns the list of slots written, in token order.
    """
    nb, B = pool.shape[0], pool.shape[1]
    slots = []
    for t in range(k_bits.shape[0]):
        s = int(token_seq[t])
        p = int(positions[t])
        blk = int(block_table[s][p // B])
        if not (0 <= blk < nb):
            raise IndexError(f"block id {blk} outside the pool of {nb} blocks")
        off = p % B
        pool[blk, off, 0] = k_bits[t]
        pool[blk, off, 1] = v_bits[t]
        slots.append(blk * B + off)
    return slots
