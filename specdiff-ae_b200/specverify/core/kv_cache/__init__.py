"""Paged KV storage (copy-on-write) and the chunk arena."""

from .chunk_arena import ChunkArena, ChunkArenaConfig, ChunkArenaWithAPW, arena_page_table
from .paged_kv import PagedKVCache, PagedKVConfig

__all__ = ["PagedKVCache", "PagedKVConfig", "ChunkArena", "ChunkArenaConfig", "ChunkArenaWithAPW",
           "arena_page_table"]
