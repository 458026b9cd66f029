"""Three-level memory network: instant (live KV sessions), short-term (sliding window
of conversation turns) and long-term (vector store with an HNSW index)."""
from .dmn import InstantMemory, LongTermMemory, MemoryManager, ShortTermMemory
from .hnsw import HNSWIndex

__all__ = ["HNSWIndex", "InstantMemory", "ShortTermMemory", "LongTermMemory", "MemoryManager"]
