"""Helpers of the special_attentions mirror."""
