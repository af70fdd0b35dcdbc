/* TEST INFRASTRUCTURE ONLY.  Stand-in for <liburing.h> (absent here) when
 * the reference's csrc/transfer_ssd.cpp is compiled as the SSD-tier oracle.
 * The oracle always opens its contexts with iouring_entries = 0, so the
 * reference takes its thread-pool path and never reaches these; should it
 * try, queue set-up fails (-ENOSYS) and the reference falls back to threads
 * as it does when the kernel refuses io_uring. */
#pragma once
#include <errno.h>
#include <sys/uio.h>

struct io_uring { int unused; };
struct io_uring_sqe { int unused; };
struct io_uring_cqe { unsigned long long user_data; int res; unsigned flags; };

static inline int io_uring_queue_init(unsigned, struct io_uring *, unsigned) { return -ENOSYS; }
static inline void io_uring_queue_exit(struct io_uring *) {}
static inline int io_uring_submit(struct io_uring *) { return -ENOSYS; }
static inline int io_uring_wait_cqe(struct io_uring *, struct io_uring_cqe **) { return -ENOSYS; }
static inline int io_uring_peek_cqe(struct io_uring *, struct io_uring_cqe **) { return -EAGAIN; }
static inline void *io_uring_cqe_get_data(const struct io_uring_cqe *) { return nullptr; }
static inline void io_uring_cqe_seen(struct io_uring *, struct io_uring_cqe *) {}
static inline struct io_uring_sqe *io_uring_get_sqe(struct io_uring *) { return nullptr; }
static inline void io_uring_prep_readv(struct io_uring_sqe *, int, const struct iovec *, unsigned, unsigned long long) {}
static inline void io_uring_prep_writev(struct io_uring_sqe *, int, const struct iovec *, unsigned, unsigned long long) {}
static inline void io_uring_sqe_set_data(struct io_uring_sqe *, void *) {}
