"""Evaluation: message perplexity, generated-vs-real order-flow statistics, return bench."""
