"""Serving-framework registration (SGLang 0.5.22, vLLM 0.26.0); inert until opted in."""
