"""Serving: a request scheduler that owns the model (prefill through the RidgeFill engine, greedy decode streams
interleaved with long prefills at layer granularity), an HTTP server with a llama.cpp-style `/completion` endpoint
(SSE streaming, per-request timings), and the measurement clients that drive it: the warm TTFT timing run and the
fixed-arrival concurrency mix (the roles of code/qwen38-27b-kit/common.py, timing.py and mix.py, which drove an
external llama.cpp server)."""
