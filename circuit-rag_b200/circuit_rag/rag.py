"""Text-in / text-out wrapper (reference circuit_rag/rag.py:11-65).

The embedding model is out of scope for the search path and sentence-
transformers is an optional dependency: CircuitRAG imports it only when it is
constructed without an ``embed_fn``.  Any callable mapping a list of strings to
a float32 [n, D] array can be passed instead.
"""
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import numpy as np
import torch

from circuit_rag.hierarchy.build import build_circuit_index
from circuit_rag.search import circuit_search


@dataclass
class SearchResult:
    id: int
    score: float
    text: str
    metadata: Dict[str, Any] = field(default_factory=dict)


class CircuitRAG:
    def __init__(self, embedding_model: str = "BAAI/bge-small-en-v1.5", device: Optional[str] = None,
                 embed_fn: Optional[Callable[[List[str]], np.ndarray]] = None):
        self.device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        if embed_fn is None:
            from sentence_transformers import SentenceTransformer  # optional dependency

            model = SentenceTransformer(embedding_model, device=self.device)
            embed_fn = lambda texts: model.encode(texts, normalize_embeddings=True, convert_to_numpy=True)
        self._embed = embed_fn
        self.texts: List[str] = []
        self.metadatas: List[Dict[str, Any]] = []
        self._vectors: Optional[np.ndarray] = None
        self.index = None

    def add_documents(self, texts: List[str], metadatas: Optional[List[Dict[str, Any]]] = None) -> List[int]:
        """Embed and add documents, then rebuild the index (as the reference does)."""
        if metadatas is None:
            metadatas = [{} for _ in texts]
        vecs = np.asarray(self._embed(list(texts)), dtype=np.float32)
        first = len(self.texts)
        self.texts.extend(texts)
        self.metadatas.extend(metadatas)
        self._vectors = vecs if self._vectors is None else np.concatenate([self._vectors, vecs])
        n = len(self._vectors)
        roots = max(1, min(64, n // 16))
        self.index = build_circuit_index(self._vectors, num_roots=roots, children_per_root=max(1, min(16, n // roots)),
                                         rank=min(8, self._vectors.shape[1]), device=self.device)
        return list(range(first, n))

    def search(self, query: str, k: int = 5) -> List[SearchResult]:
        if self.index is None:
            return []
        q = torch.from_numpy(np.asarray(self._embed([query]), dtype=np.float32)[0])
        scores, ids, _ = circuit_search(q, self.index, k=min(k, len(self.texts)))
        return [SearchResult(id=int(i), score=float(s), text=self.texts[int(i)], metadata=self.metadatas[int(i)])
                for s, i in zip(scores.tolist(), ids.tolist())]
