"""sm_100a operators behind the reference's attention-backend API."""
