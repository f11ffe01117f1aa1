// Declarations shared by the translation units of libtgcb.so; not part of the C-ABI.
#ifndef TGCB_INTERNAL_H_
#define TGCB_INTERNAL_H_

// Devices the library tracks per process (device ordinals 0 .. kTgcbMaxDevices-1). Every entry
// point that keeps per-device state accepts exactly this range.
constexpr int kTgcbMaxDevices = 16;

// Records the calling thread's last error (runtime.cu) and returns `code`.
int tgcb_internal_fail(int code, const char* what, const char* detail);

// Looks up and stores the device address of the allocation-free pairwise sum's scratch array
// for the current device (reductions.cu). tgcb_init calls it with the device current, on every
// call, so a re-initialised context gets a fresh address. The lookup may load the library's
// module on that device (lazy loading), which is when the driver places the array.
int tgcb_internal_noalloc_setup(int device);

// The current device's status word (initialising the device's state on first use), for
// kernels launched outside a plan that report device-side failures the way plans do.
int tgcb_internal_status_word(int** out);

#endif  // TGCB_INTERNAL_H_
