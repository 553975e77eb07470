"""Operators of the decode hot path: skinny linear and the fused mLSTM recurrence."""
