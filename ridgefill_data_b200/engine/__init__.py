"""RidgeFill prefill engine over the per-layer model API (arms, layer-major prefill, decode, scoring)."""
