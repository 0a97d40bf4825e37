"""Retrieval: TF-IDF + product-quantised index, entity graph retrieval (GraphRAG-style), logit biasing."""
from .pq import PQRetriever
from .graph import GraphRAG, logit_bias_from_text

__all__ = ["PQRetriever", "GraphRAG", "logit_bias_from_text"]
