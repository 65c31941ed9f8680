"""ridgefill_data_b200: a Blackwell-native (sm_100a) long-prompt prefill engine with RidgeFill.

Layers below a split S run exactly; every later layer fills its cache (attention K/V, or the
Gated DeltaNet conv and recurrent state) from a closed-form ridge prediction of its input,
x_l = h_S W_l^T + c_l; the last T prompt rows and every decode step run the full model.
"""
__version__ = "0.1.0"
