"""lightbulb_b200: a Blackwell (B200, sm_100a) native LLM inference engine and server.

Public entry points:

* :class:`lightbulb_b200.engine.llm_engine.LLMEngine` - continuous-batching engine
* :class:`lightbulb_b200.engine.sampling.SamplingParams`
* ``python -m lightbulb_b200.cli.serve`` - OpenAI-compatible HTTP server
* ``python -m lightbulb_b200.cli.local_gen`` - CPU ``local-llama-gen`` path
"""
__version__ = "0.1.0"
