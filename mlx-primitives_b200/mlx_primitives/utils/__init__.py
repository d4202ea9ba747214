"""Helpers of the attention path."""
