"""Process-free test doubles (see ``dist_doubles``)."""
