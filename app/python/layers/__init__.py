"""Drop-in names for the reference's app/python/layers package."""
