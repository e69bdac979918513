"""Evaluation: frozen suites, clients (Inspect AI, EuroEval, direct OpenAI-compatible, CPU fixture), metrics."""
