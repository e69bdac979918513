"""Serving exported Mimir2 models through an OpenAI-compatible vLLM server."""
