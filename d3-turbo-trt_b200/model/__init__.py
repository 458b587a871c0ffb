"""Operators under d3trt/model: W8A8 Linear, attention dispatch, readout."""
