// Link search path for libmoe_b200.so (built by `python moe-680m_b200/build.py`); override with
// MOE_B200_LIB_DIR.
fn main() {
    let dir = std::env::var("MOE_B200_LIB_DIR").unwrap_or_else(|_| {
        let here = std::env::var("CARGO_MANIFEST_DIR").unwrap();
        format!("{}/../moe-680m_b200/lib", here)
    });
    println!("cargo:rustc-link-search=native={}", dir);
    println!("cargo:rustc-link-lib=dylib=moe_b200");
    println!("cargo:rerun-if-env-changed=MOE_B200_LIB_DIR");
}
