"""Comparison backends: a stock serving engine asked one request per row.

These exist to measure this engine against; a user runs the `quail` backend.
`vllm_backend.VLLMEngine` answers a region's calls by sending every row's
whole prompt (instruction prefix, document, question) to vLLM as its own
request, with vLLM's prefix caching on, and reading the answer tokens' log
probabilities of one generated token (the reference's stock-vLLM request
backend, quail/baselines/vllm.py and request.py). `hf_export` writes the
random-init weights of a model config as a Hugging Face checkpoint directory
vLLM can load, so both engines run the same network. `bench` times the
flagship AI.IF workload through it.
"""


def register_baselines(registry) -> None:
    """Add the comparison backends to an extension registry (backend name -> engine factory)."""
    from quail_b200.baselines.vllm_backend import VLLMEngine
    registry.register_backend("vllm", VLLMEngine)
