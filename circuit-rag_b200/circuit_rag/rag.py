"""Text-in / text-out wrapper (reference circuit_rag/rag.py:11-65), with
incremental document adds instead of a full rebuild per call.

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
        self._built_n = 0
        self.appended_rows = 0

    # appended rows beyond this fraction of the last full build trigger a rebuild
    REBUILD_FRACTION = 0.5

    def add_documents(self, texts: List[str], metadatas: Optional[List[Dict[str, Any]]] = None) -> List[int]:
        """Embed and add documents; returns their ids (reference rag.py:33-45).

        The reference rebuilds the whole index on every call.  Here new
        documents are appended to the existing hierarchy (CircuitIndex.append:
        nearest root, new child, certificates recomputed) until the appended
        rows exceed REBUILD_FRACTION of the rows of the last full build; then
        the index is rebuilt with the reference's size rule (rag.py:47-55)."""
        texts = list(texts)
        if metadatas is None:
            metadatas = [{} for _ in range(len(texts))]
        elif len(metadatas) != len(texts):
            raise ValueError("metadatas must be the same length as texts")
        new_vecs = np.asarray(self._embed(texts), dtype=np.float32)
        start_id = len(self.texts)
        self.texts.extend(texts)
        self.metadatas.extend(metadatas)
        if self._vectors is None:
            self._vectors = new_vecs
        else:
            self._vectors = np.concatenate([self._vectors, new_vecs], axis=0)
        n = len(self._vectors)
        if self.index is not None and (n - self._built_n) <= self.REBUILD_FRACTION * self._built_n:
            self.index.append(new_vecs, np.arange(start_id, n, dtype=np.int32))
            self.appended_rows = n - self._built_n
        else:
            self._rebuild()
        return list(range(start_id, n))

    def _rebuild(self):
        n = len(self._vectors)
        roots = int(max(1, min(64, n // 256)))
        children = int(max(1, min(16, n // (roots * 16))))
        self.index = build_circuit_index(self._vectors, num_roots=roots, children_per_root=children,
                                         rank=min(8, self._vectors.shape[1]), device=self.device)
        self._built_n = n
        self.appended_rows = 0

    def search(self, query: str, k: int = 5) -> List[SearchResult]:
        if self.index is None:
            return []
        q = torch.from_numpy(np.asarray(self._embed([query]), dtype=np.float32)[0])
        scores, ids, _ = circuit_search(q, self.index, k=min(k, len(self.texts)))
        return [SearchResult(id=int(i), score=float(s), text=self.texts[int(i)], metadata=self.metadatas[int(i)])
                for s, i in zip(scores.tolist(), ids.tolist())]
