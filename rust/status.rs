// Status check for src/lib.rs's two FFI call sites (the reference returns Ok(()) even when its
// kernels fail to launch).  Add `mod status;` to lib.rs and call
//
//     unsafe { ffi::topk_softmax(...) }
//     status::check("topk_softmax")?;          // after src/lib.rs:108-119
//
//     unsafe { ffi::fused_moe(...) }
//     status::check("fused_moe")?;             // after src/lib.rs:450-469
//
// Not compiled in the image this library was built in (no cargo there): unverified.
use crate::ffi;
use std::ffi::CStr;

/// Err with the library's description when the last drop-in call of this thread failed.
pub(crate) fn check(what: &str) -> candle::Result<()> {
    let st = unsafe { ffi::moe_last_status() };
    if st == 0 {
        return Ok(());
    }
    let msg = unsafe { CStr::from_ptr(ffi::moe_status_string(st)) };
    candle::bail!("{what} failed: {} (status {st})", msg.to_string_lossy())
}
