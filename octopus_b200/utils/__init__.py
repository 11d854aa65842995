"""Utilities: transfer accounting, timing, logging."""
