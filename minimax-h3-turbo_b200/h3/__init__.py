"""Drop-in counterparts of the reference's `h3turbo.h3` modules for the W4A8 hot path (qlinear, types, and the weight
store / streamer that feed it)."""
